// C ABI of the tcgen05 GEMM (no PyTorch types; callable from any host code).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

struct GemmParams {
  int rows_p, rows_q;
  int tiles_p, tiles_q;
  int splits, kb_total, kb_per_split;
  __nv_bfloat16* out;
  int ldo;
  float* ws;
  int* err;
  int p_fast;
};

#ifdef __cplusplus
extern "C" {
#endif
// D[i, j] = sum_k P[i, k] Q[j, k] (bf16 in, fp32 accumulate, bf16 out).
//   trans = 0: out[i * ldo + j];  trans = 1: out[j * ldo + i].
//   bn in {64, 128, 256}: Q tile rows (MMA N).  splits > 1 needs a workspace
//   ws of splits * rows_p * rows_q floats.  err (optional) receives a
//   non-zero code if a pipeline wait timed out.  Returns 0 on success.
int sh_gemm_bf16_tcgen05(const void* P, int rows_p, int64_t ldp, const void* Q, int rows_q, int64_t ldq, int K,
                         void* out, int64_t ldo, int trans, int bn, int splits, float* ws, int* err, int num_sms,
                         cudaStream_t stream);
#ifdef __cplusplus
}
#endif
