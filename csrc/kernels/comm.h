// C ABI of the NVLink symmetric-memory collectives (no PyTorch types).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define SH_COMM_MAX_WORLD 8
#define SH_COMM_MAX_BLOCKS 160

struct ArParams {
  // Per-rank symmetric buffers (device addresses valid in this process).
  const __nv_bfloat16* peer_in[SH_COMM_MAX_WORLD];  // [T, H] partial sums (this rank's entry is local)
  __nv_bfloat16* peer_gather[SH_COMM_MAX_WORLD];    // [T, H] two-shot gather buffers
  uint32_t* peer_flags[SH_COMM_MAX_WORLD];          // signal pads
  uint32_t* counters;                               // [SH_COMM_MAX_BLOCKS] local epoch counters
  __nv_bfloat16* residual;                          // [T, H] (fused norm) or nullptr
  __nv_bfloat16* out;                               // [T, H]: normed x (fused) or the sum
  const __nv_bfloat16* weight;                      // [H] RMSNorm weight (fused)
  int* err;                                         // timeout report (code, nonzero on failure)
  int rank, world;
  int T, H;
  float eps;
  int two_shot;
  int fuse_norm;
};

#ifdef __cplusplus
extern "C" {
#endif
// Sum of the world ranks' [T, H] partials, optionally fused with
// residual += sum; out = rms_norm(residual) * weight.  All ranks must call it
// with identical T, H, mode and grid in the same order.  Returns 0 on launch.
int sh_allreduce(const ArParams* p, int num_blocks, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
