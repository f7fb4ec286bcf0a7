// C ABI of the MoE routing / movement kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

struct RouteParams {
  const void* logits;  // [T, E] router logits (fp32 or bf16)
  int logits_bf16;
  const float* bias;  // [E] selection bias (sigmoid_grouped) or nullptr
  int32_t* ids;       // [T, k]
  float* weights;     // [T, k]
  int T, E, k;
  int sigmoid_grouped;  // 0: softmax top-k; 1: sigmoid, group-limited
  int n_groups, topk_groups;
  int renorm;
  float scale;
};

struct AlignParams {
  const int32_t* ids;     // [T, k]
  int32_t* rank;          // [T*k] scratch: rank within the expert
  int32_t* offsets;       // [E+1]
  int32_t* sorted_pos;    // [T*k]: sorted row of pair (t, j) (-1 if dropped)
  int32_t* sorted_token;  // [T*k]: token of each sorted row
  int4* groups;           // [max_groups] {row0, rows, expert weight row offset, expert}
  int* num_groups;        // [1]
  int T, k, E, bn, max_groups, rows_per_expert;
};

#ifdef __cplusplus
extern "C" {
#endif
int sh_moe_route(const RouteParams* p, cudaStream_t stream);
int sh_moe_align(const AlignParams* p, cudaStream_t stream);
int sh_moe_gather(__nv_bfloat16* out, const __nv_bfloat16* x, const int32_t* sorted_token, const int* total,
                  int max_rows, int H, cudaStream_t stream);
int sh_moe_combine(__nv_bfloat16* out, const __nv_bfloat16* y, const int32_t* sorted_pos, const float* w, int T, int k,
                   int H, int accumulate, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
