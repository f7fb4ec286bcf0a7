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
  int p_is_weight;  // P holds the weights (read once: L2 evict-first), Q the activations (evict-last); else swapped
  // Grouped (MoE) mode when groups != nullptr: work unit = (group entry, P
  // tile).  Entry = {q_row0, q_rows, p_row_offset, unused}: the Q tile starts at
  // sorted row q_row0 and holds q_rows valid rows; P tiles start at row
  // p_row_offset (the expert's first weight row) and span rows_p rows.
  const int4* groups;
  const int* num_groups;
  // Reduce-scatter push (row-parallel GEMM under tensor parallelism, push != 0):
  // output row t (a token) is stored into rank o = t / push_rows's receive slot
  // push_recv[o] + ((par * push_world + push_rank) * push_max_T + t) * N + n
  // (N = the output width, par = parity of the next comm call = (*push_epoch + 1) & 1),
  // and after each tile every epilogue warp adds 1, with release semantics, to
  // push_cnt[o][par] of every owner o whose token rows it stored (non-TRANS:
  // the warp's 32 rows of the tile; TRANS: the tile's token columns).
  int push;
  __nv_bfloat16* push_recv[8];
  uint32_t* push_cnt[8];
  const uint32_t* push_epoch;
  int push_rank, push_world, push_rows, push_max_T, push_n;
};

// Stream-K linear on CTA pairs (gemm_streamk.cu): y[j, i] = sum_k W[i, k] X[j, k].
struct SkParams {
  int rows_w, rows_x;
  int tiles_w, tiles_x;  // 256-row weight tiles x NT-token tiles; tile = tw * tiles_x + tx
  int kb;                // 64-wide k-blocks per tile
  int clusters;          // CTA pairs launched
  int q;                 // whole tiles per cluster: cluster c owns tiles [c*q, c*q + q)
  int64_t sk_iters;      // k-blocks of the split tiles (tiles % clusters of them, after the whole ones)
  int sk_clusters;       // clusters sharing the split k-blocks evenly (their pieces run first)
  float* ws;             // fp32 partial slots [clusters][2 ranks][2][NT][128]
  int* cnt;              // [tiles][2] arrival counters, zero between calls
  int* err;
  // Optional phase timestamps (%globaltimer ns) per CTA, [grid][64] (nullptr: off); see gemm_streamk.cu.
  unsigned long long* stamps;
  __nv_bfloat16* y;      // output [rows_x][ldy]
  int64_t ldy;
};

#ifdef __cplusplus
extern "C" {
#endif
// Stream-K linear y = X W^T on tcgen05 CTA pairs, weights on the MMA M side:
// W [rows_w, K] (row stride ldw), X [rows_x, K], y [rows_x, ldy] bf16; K % 64 == 0,
// 16-byte aligned bases and row strides, rows_w % 8 == 0.  One tile = 256 weight rows x
// ns*nsub tokens ((ns, nsub) in {(64,1), (128,1), (192,1), (256,1), (192,2), (256,2)}).
// `clusters` CTA pairs each own tiles / clusters whole tiles and share the
// k-blocks of the remaining tiles (a split tile has at most 3 pieces).  ws: >= the floats reported by
// sh_gemm_sk_shape; cnt: >= 2 * tiles ints, zero before the first call (the
// kernel leaves them zero).  One call at a time per (ws, cnt) pair.
int sh_gemm_bf16_sk(const void* W, int rows_w, int64_t ldw, const void* X, int rows_x, int64_t ldx, int K, void* Y,
                    int64_t ldy, int ns, int nsub, int clusters, float* ws, int* cnt, int* err,
                    unsigned long long* stamps, cudaStream_t stream);
// Tile count and workspace floats of a stream-K call (0 on success).
int sh_gemm_sk_shape(int rows_w, int rows_x, int K, int ns, int nsub, int clusters, int64_t* tiles,
                     int64_t* ws_floats);
// Co-resident CTA pairs of the stream-K kernel on the current device.
int sh_gemm_sk_max_clusters(int ns, int nsub);
// D[i, j] = sum_k P[i, k] Q[j, k] (bf16 in, fp32 accumulate, bf16 out).
//   trans = 0: out[i * ldo + j];  trans = 1: out[j * ldo + i].
//   bn in {64, 128, 256}: Q tile rows (MMA N).  splits > 1 needs a workspace
//   ws of splits * rows_p * rows_q floats.  err (optional) receives a
//   non-zero code if a pipeline wait timed out.  Returns 0 on success.
int sh_gemm_bf16_tcgen05(const void* P, int rows_p, int64_t ldp, const void* Q, int rows_q, int64_t ldq, int K,
                         void* out, int64_t ldo, int trans, int bn, int splits, float* ws, int* err, int num_sms,
                         cudaStream_t stream);
// Same contract on CTA pairs (cta_group::2, 256-row P tiles; bn in {128, 192, 256}).
int sh_gemm_bf16_pair(const void* P, int rows_p, int64_t ldp, const void* Q, int rows_q, int64_t ldq, int K,
                      void* out, int64_t ldo, int trans, int bn, int splits, float* ws, int* err, int num_sms,
                      cudaStream_t stream);
// Row-parallel GEMM whose epilogue pushes output rows to their owner ranks (see
// GemmParams::push*).  P holds the token rows (trans = 0 only), splits = 1;
// pair selects the CTA-pair kernel (bn 128/192/256) over the one-CTA kernel
// (bn 64/128/256).  `push` holds the push fields (other members ignored).
int sh_gemm_bf16_push(const void* P, int rows_p, int64_t ldp, const void* Q, int rows_q, int64_t ldq, int K,
                      int trans, int bn, int pair, const GemmParams* push, int* err, int num_sms,
                      cudaStream_t stream);
// Grouped swap-AB GEMM for MoE experts: for every device-side group entry g
// (see GemmParams::groups), out[q, :] = sum_k Q[q, k] * P[p_row_offset + n, k]
// for the q_rows sorted rows of the entry and n < rows_p.  P stacks the
// experts' [rows_p, K] weights; Q holds the expert-sorted activations
// [q_total, K]; out is [q_total, ldo].  max_groups bounds the list length.
int sh_gemm_bf16_grouped(const void* P, int p_total_rows, int rows_p, const void* Q, int q_total, int K, void* out,
                         int64_t ldo, const int4* groups, const int* num_groups, int max_groups, int bn, int* err,
                         int num_sms, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
