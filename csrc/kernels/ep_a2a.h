// C ABI of the expert-parallel all-to-all over NVLink peer memory (no PyTorch types).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "moe.h"

#define SH_EP_MAX_WORLD 8
#define SH_EP_MAX_BLOCKS 160
#define SH_EP_MAX_K 16

// One call = dispatch, the expert GEMMs on the received rows, combine.  Every
// rank holds T tokens (T equal on every rank within a call).  Received rows
// are laid out by source rank: rows [r*T, r*T + T) of a receive buffer hold
// source rank r's tokens, so the expert GEMMs see one [world*T, H] matrix.
struct EpParams {
  const __nv_bfloat16* x;                  // [T, H] this rank's tokens (dispatch)
  const int32_t* ids;                      // [T, k] global expert ids of this rank's tokens
  const float* w;                          // [T, k] route weights (dispatch)
  __nv_bfloat16* peer_x[SH_EP_MAX_WORLD];  // per rank: [world*max_T][H] received token rows
  int32_t* peer_ids[SH_EP_MAX_WORLD];      // per rank: [world*max_T][k] local expert id, -1 elsewhere
  float* peer_w[SH_EP_MAX_WORLD];          // per rank: [world*max_T][k] weight, 0 elsewhere
  const __nv_bfloat16* y;                  // combine: [world*T, H] this rank's expert outputs per received row
  __nv_bfloat16* peer_y[SH_EP_MAX_WORLD];  // per rank: [world*max_T][H] returned rows, rows [d*T, d*T+T) from rank d
  __nv_bfloat16* out;                      // combine: [T, H] sum over the expert ranks in rank order
  uint32_t* peer_flags[SH_EP_MAX_WORLD];   // per rank: [2 phases][SH_EP_MAX_BLOCKS][SH_EP_MAX_WORLD]
  uint32_t* counters;                      // [SH_EP_MAX_BLOCKS] local epochs (dispatch advances them)
  int* err;                                // nonzero after a timed-out wait (200 + barrier phase)
  unsigned long long wait_ns;              // limit of each cross-rank wait in ns (0: the default, 5 s)
  int rank, world, T, H, k, e_local, max_T;
  // quant = 1: the dispatch quantises each row to NVFP4 once (per-row g = 2688 / amax, e4m3 scale per 16,
  // e2m1 codes: the activation quantiser's math) and sends codes, scales and 1 / g instead of bf16 rows.
  int quant;
  uint8_t* peer_q[SH_EP_MAX_WORLD];  // per rank: [world*max_T][H/2] e2m1 codes
  uint8_t* peer_s[SH_EP_MAX_WORLD];  // per rank: [world*max_T][H/16] e4m3 scales
  float* peer_a[SH_EP_MAX_WORLD];    // per rank: [world*max_T] 1 / g
  // fused_route = 1: the dispatch routes its own tokens from the router logits (route.logits [T, E]) with
  // the standalone router's selection and writes route.ids / route.weights [T, k] (ids must equal
  // route.ids: the combine reads them); `w` is then unused.
  int fused_route;
  RouteParams route;
  // Combine fused with the experts' weighted per-token sum (sh_ep_combine_push): row r*T + i of the
  // received rows = sum_j w_local[row, j] * ys[sorted_pos[row * k + j]] (pairs with sorted_pos < 0 skipped),
  // stored straight into owner r's return rows; sh_ep_combine with pushed = 1 then only meets and sums.
  const __nv_bfloat16* ys;   // [pairs][H] expert outputs in sorted pair order
  const int32_t* sorted_pos;  // [world*T][k]
  const float* w_local;       // [world*T][k] local route weights (0 for other ranks' experts)
  int pushed;
};

#ifdef __cplusplus
extern "C" {
#endif
// Both use the same grid on every rank and for every call of a communicator.
int sh_ep_dispatch(const EpParams* p, int num_blocks, cudaStream_t stream);
int sh_ep_combine(const EpParams* p, int num_blocks, cudaStream_t stream);
int sh_ep_combine_push(const EpParams* p, int num_blocks, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
