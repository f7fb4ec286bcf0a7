// C ABI of the block-scaled NVFP4 (W4A4) tcgen05 GEMM and its activation quantiser.
//
// Scale-factor tiles ("sf tiles"): the e4m3 block scales of 128 rows of a
// matrix, for every 64 consecutive k (four 16-element blocks), are one 512-byte
// chunk in the tensor-core layout: byte (r % 32) * 16 + (r / 32) * 4 + (k / 16) % 4
// for row r of the tile.  A tile stores kc4 = round_up(K / 64, 4) chunks in k
// order (chunks past K / 64 are zero), so one 256-wide k-block reads 2 KB.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

struct Fp4MmaParams {
  const uint8_t* w;             // [rows_total, K/2] packed e2m1 weights (low nibble = even k)
  const uint8_t* w_sf;          // [num_matrices * tiles_p][kc4][512] weight scale tiles (per matrix)
  const float* alpha_w;         // [1] (dense) or [E] (grouped): weight global dequantisation scale
  const uint8_t* x_sf;          // [q tiles][kc4][512] activation scale tiles (dense: tile t = rows t*bn..;
                                //   grouped: one tile per group entry)
  const float* a_scale;         // [rows_q] per-token activation dequantisation scale
  __nv_bfloat16* out;           // [rows_q, ldo]: out[token, weight row within its matrix]
  int64_t ldo;
  int rows_total;               // stacked weight rows
  int rows_p;                   // rows per weight matrix (grouped: per expert; dense: rows_total)
  int K;
  int rows_q, tiles_p, tiles_q;  // filled by the launcher
  int splits, kb_per_split;      // split-K (dense mode): fp32 partial tiles in ws; the last split of a
                                 // tile (ticket in counters) sums them in split order and stores
  float* ws;                     // [splits][tiles_p * tiles_q][128][bn]
  int* counters;                 // [tiles_p * tiles_q] zero before the first launch; re-armed by the kernel
  int out_vec;                   // filled by the launcher: 16-byte output stores allowed
  int* err;
  const int4* groups;            // grouped (MoE) entries {q_row0, q_rows, p_row_offset, expert} or nullptr
  const int* num_groups;
  int max_groups;
  unsigned long long* stamps;    // optional per-CTA timings, ns ([grid][8]; profiling): setup, PDL wait, first
                                 // stage landed, first accumulator ready, accumulator waits, split partial
                                 // writes + ticket, reduce + store, whole CTA
};

#ifdef __cplusplus
extern "C" {
#endif
// NVFP4 quantisation of bf16 activations x [rows, K] (row stride ldx):
//   g_r = static_g if static_g > 0 else 2688 / amax(|x_r|) (1 for an all-zero row);
//   block scale s = e4m3(amax16 * g_r / 6); code = e2m1_rne(x * (g_r / s));
//   xq [rows, K/2] packed codes; a_scale[r] = 1 / g_r; scales into the sf tile of
//   the row: dense (groups == nullptr): tile r / tile_rows, slot r % tile_rows;
//   grouped: the entry e with q_row0 <= r < q_row0 + q_rows, slot r - q_row0.
// max_tiles bounds the grid (dense: ceil(rows / tile_rows); grouped: max_groups).
// swiglu: x rows are a fused gate | up projection [2K] (row stride ldx >= 2K) and the quantised
// activation is silu(gate) * up (bf16-rounded), i.e. the SwiGLU is fused into the quantiser.
int sh_nvfp4_quant_act(const void* x, int64_t ldx, int rows, int K, const int4* groups, const int* num_groups,
                       int max_tiles, int tile_rows, float static_g, uint8_t* xq, uint8_t* x_sf, float* a_scale,
                       int swiglu, cudaStream_t stream);
// Pre-quantised NVFP4 rows (codes [*, K/2], e4m3 scales [*, K/16], a_scale [*]) gathered by token[r] into
// the grouped operand layout of rows [0, rows) (the layout sh_nvfp4_quant_act writes with groups).
int sh_nvfp4_gather_act(const uint8_t* codes, const uint8_t* scales, const float* ascale, const int* token, int rows,
                        int K, const int4* groups, const int* num_groups, uint8_t* xq, uint8_t* x_sf, float* a_scale,
                        cudaStream_t stream);
// out[t, n] = alpha_w * a_scale[t] * sum_k e2m1(xq[t, k]) sx(t, k) e2m1(w[n, k]) sw(n, k); bn in {64, 128}.
// splits > 1 (dense mode) needs ws (splits * tiles_p * tiles_q * 128 * bn floats) and zeroed counters.
int sh_gemm_fp4mma(Fp4MmaParams* g, const void* xq, int rows_q, int bn, int splits, int num_sms,
                   cudaStream_t stream);
// MXFP8 (W8A8) on the same kernel: w [rows_total, K] e4m3, w_sf / x_sf tiles of ue8m0 scales per 32 values
// (chunk c covers k 128c .. 128c+127; byte (r % 32) * 16 + (r / 32) * 4 + (k / 32) % 4), K % 128 == 0.
int sh_gemm_mxfp8(Fp4MmaParams* g, const void* xq, int rows_q, int bn, int splits, int num_sms,
                  cudaStream_t stream);
// bf16 activations -> e4m3 codes xq [rows, K] with ue8m0 scales per 32 values (scale tiles as above);
// a_scale[r] = 1.  Grouped rows map to their entry's tile like sh_nvfp4_quant_act.
int sh_mxfp8_quant_act(const void* x, int64_t ldx, int rows, int K, const int4* groups, const int* num_groups,
                       int tile_rows, uint8_t* xq, uint8_t* x_sf, float* a_scale, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
