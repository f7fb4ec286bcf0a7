// C ABI of the NVLink symmetric-memory collectives (no PyTorch types).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define SH_COMM_MAX_WORLD 8
#define SH_COMM_MAX_BLOCKS 160
#define SH_COMM_PHASES 2

struct ArParams {
  const __nv_bfloat16* partial;                    // [T, H] this rank's partial sum (local memory)
  __nv_bfloat16* peer_recv[SH_COMM_MAX_WORLD];     // per rank: [2][world][max_T][H] receive slots
  __nv_bfloat16* peer_gather[SH_COMM_MAX_WORLD];   // per rank: [2][max_T][H] reduced rows (two-shot)
  uint32_t* peer_flags[SH_COMM_MAX_WORLD];         // per rank: [SH_COMM_PHASES][SH_COMM_MAX_BLOCKS][MAX_WORLD]
  uint32_t* counters;                              // [SH_COMM_MAX_BLOCKS] local epoch counters
  __nv_bfloat16* residual;                         // [T, H] (fused norm) or nullptr
  __nv_bfloat16* out;                              // [T, H]: normed x (fused) or the sum
  const __nv_bfloat16* weight;                     // [H] RMSNorm weight (fused)
  int* err;                                        // timeout report (code, nonzero on failure)
  int rank, world;
  int T, H, max_T;
  float eps;
  int two_shot;
  int fuse_norm;
  // Optional phase timestamps (%globaltimer, ns) of block 0: [64 calls][4] =
  // entry, pushes issued, first wait passed, exit; slot = epoch % 64.
  unsigned long long* timing;
};

#ifdef __cplusplus
extern "C" {
#endif
// Sum of the world ranks' [T, H] partials, optionally fused with
// residual += sum; out = rms_norm(residual) * weight.  All ranks must call it
// with identical T, H, mode and grid (every call of a communicator uses the
// same grid) in the same order.  Returns 0 on launch.
int sh_allreduce(const ArParams* p, int num_blocks, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
