// C ABI of the NVLink symmetric-memory collectives (no PyTorch types).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define SH_COMM_MAX_WORLD 8
#define SH_COMM_MAX_BLOCKS 160
#define SH_COMM_PHASES 3

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
  // Optional L2 prefetch of the next GEMM's weights while the ranks wait on
  // each other (every block takes a slice; nullptr / 0 = none).
  const void* prefetch;
  unsigned long long prefetch_bytes;
  // Limit of each cross-rank wait in ns (0: the default, 5 s).  On expiry the
  // kernel records 100 + phase in *err and returns.
  unsigned long long wait_ns;
  // Compressed transfer (H % 128 == 0): 0 = bf16 rows; 1 = int8, 2 = fp8 e4m3 codes with one fp32 scale
  // per 128 elements (amax / 127 or amax / 448), a row packed as [H codes | H / 128 scales] in its bf16
  // slot.  Every rank sums the same dequantised bytes in rank order, so the results stay bit-identical;
  // the two-shot form requantises the owner's sum for the gather (two roundings, like the reference).
  int quant;
};

// Reduce-scatter tail of a row-parallel GEMM whose epilogue pushed its output
// rows into the owners' receive slots (GemmParams::push): the owner waits until
// `expected` tile arrivals were counted on rs_cnt[par], sums its rows in rank
// order, residual += sum, y = rms_norm(residual) * weight, and pushes y (and,
// with gather_res, the residual rows) to every rank's gather buffer; after a
// cross-rank barrier every rank copies all T rows into out (and residual).
struct RsParams {
  const __nv_bfloat16* recv;                          // this rank's receive buffer [2][world][max_T][H]
  __nv_bfloat16* peer_gather[SH_COMM_MAX_WORLD];      // per rank: [2][max_T][H] normalised rows
  __nv_bfloat16* peer_gather_res[SH_COMM_MAX_WORLD];  // per rank: [2][max_T][H] residual rows
  uint32_t* peer_flags[SH_COMM_MAX_WORLD];            // per rank: barrier flags (phase 2)
  uint32_t* rs_cnt;                                   // this rank's arrival counters [2]
  uint32_t* targets;                                  // [SH_COMM_MAX_BLOCKS][2] running targets (block-local)
  uint32_t* counters;                                 // [SH_COMM_MAX_BLOCKS] epochs (shared with sh_allreduce)
  __nv_bfloat16* residual;                            // [T, H]: owned rows updated; all rows with gather_res
  __nv_bfloat16* out;                                 // [T, H] normalised rows
  const __nv_bfloat16* weight;                        // [H]
  int* err;
  int rank, world;
  int T, H, max_T, Tc;
  uint32_t expected;
  float eps;
  int gather_res;
  unsigned long long* timing;  // optional [64][4] phase stamps of block 0
  const void* prefetch;        // optional L2 prefetch of the next GEMM's weights (as ArParams)
  unsigned long long prefetch_bytes;
  unsigned long long wait_ns;  // wait limit (0: 5 s); 200 = arrivals, 102 = the gather barrier
};

// Vocab-parallel greedy argmax in one kernel: every rank reduces each row of
// its logits slice to a (value, global id) key, stores the key into every
// peer's key slots, meets the peers at a same-block barrier and takes the best
// key over the ranks (max value, lowest id on ties; the key order makes one
// unsigned max do both).  Keys are double-buffered by epoch parity like the
// all-reduce's receive slots.
struct ArgmaxParams {
  const __nv_bfloat16* logits;                     // [T, V_local] (row stride ld)
  int64_t ld;
  unsigned long long* peer_keys[SH_COMM_MAX_WORLD];  // per rank: [2][world][max_T] keys
  uint32_t* peer_flags[SH_COMM_MAX_WORLD];         // per rank: [SH_COMM_MAX_BLOCKS][MAX_WORLD] flags
  uint32_t* counters;                              // [SH_COMM_MAX_BLOCKS] local epoch counters
  int64_t* out;                                    // [T] global token ids
  int* err;
  int rank, world;
  int T, V_local, max_T;
  int64_t vocab_offset;
  unsigned long long wait_ns;  // wait limit (0: 5 s); expiry records 100 in *err
};

#ifdef __cplusplus
extern "C" {
#endif
// Launch of the fused argmax (every call of a communicator uses the same grid).
int sh_argmax_tp(const ArgmaxParams* p, int num_blocks, cudaStream_t stream);
// Sum of the world ranks' [T, H] partials, optionally fused with
// residual += sum; out = rms_norm(residual) * weight.  All ranks must call it
// with identical T, H, mode and grid (every call of a communicator uses the
// same grid) in the same order.  Returns 0 on launch.
int sh_allreduce(const ArParams* p, int num_blocks, cudaStream_t stream);
// Launch of the reduce-scatter tail (same grid as every sh_allreduce call).
int sh_rs_norm_ag(const RsParams* p, int num_blocks, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
