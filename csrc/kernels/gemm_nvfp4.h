// C ABI of the NVFP4-weight (W4A16) tcgen05 GEMM.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

struct Fp4GemmParams {
  const uint8_t* packed;       // [rows_total, K/2] two e2m1 codes per byte (low nibble first)
  const uint8_t* scales;       // [K/64][rows_pad][4] e4m3 block scales, k-block major (rows_pad = rows_total
                               // rounded up to 128): one contiguous 512-byte run per k-block and 128-row tile
  const float* global_scale;   // [1] (dense) or [E] (grouped, indexed by the entry's expert)
  __nv_bfloat16* out;          // [rows_q, ldo]: out[token, weight row (within its matrix)]
  int64_t ldo;
  int rows_total;              // stacked weight rows
  int rows_pad;
  int K;
  int rows_q, tiles_p, tiles_q;  // filled by the launcher
  int splits, kb_per_split;      // split-K (dense mode): fp32 partials in ws, summed in split order
  float* ws;                     // [splits][rows_q][rows_total] when splits > 1
  int* err;
  // grouped (MoE) mode when groups != nullptr: entries {q_row0, q_rows, p_row_offset, expert}
  const int4* groups;
  const int* num_groups;
  int max_groups;
  int rows_p;                  // rows per expert matrix (grouped mode)
};

#ifdef __cplusplus
extern "C" {
#endif
// out[t, n] = global * sum_k x[t, k] * e2m1(packed[n, k]) * e4m3(scales[n, k/16]); bn in {64, 128, 256}.
// splits > 1 (dense mode only) needs g->ws with splits * rows_q * rows_total floats.
int sh_gemm_nvfp4(Fp4GemmParams* g, const void* x, int rows_q, int64_t ldx, int bn, int splits, int num_sms,
                  cudaStream_t stream);
#ifdef __cplusplus
}
#endif
