// C ABI of the paged attention kernel (no PyTorch types).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

struct AttnParams {
  __nv_bfloat16* out;         // [T, hq*D] (row stride out_stride elements)
  int64_t out_stride;
  const __nv_bfloat16* q;     // rows of the QKV projection: [T, >= hq*D] (row stride q_stride)
  int64_t q_stride;
  const __nv_bfloat16* k_cache;  // [num_blocks, hk, 64, D]
  const __nv_bfloat16* v_cache;
  const int32_t* block_tables;   // [B, bt_stride]
  int64_t bt_stride;
  const int64_t* seq_lens;       // [B] length including the new tokens
  const int64_t* q_start;        // [B+1]
  const int32_t* tile_req;       // [ntiles] request of each 64-row query tile
  const int32_t* tile_row0;      // [ntiles] first packed row of the tile
  float* part_o;                 // [T*hq*nsplit, D] split partials (nsplit > 1)
  float* part_ml;                // [T*hq*nsplit, 2]
  int* err;                      // optional timeout report
  int64_t num_tokens;
  int hq, hk, nsplit;
  float scale_log2;
};

#ifdef __cplusplus
extern "C" {
#endif
// Returns 0 on success; head_dim in {64, 128, 256}; block size 64.  max_rows:
// the most valid rows any query tile holds (<= 64); tiles of <= 16 / 32 rows
// let 4 / 2 warps share one row block's pages by key range.
int sh_paged_attention(const AttnParams* params, int ntiles, int num_blocks, int head_dim, int max_rows,
                       cudaStream_t stream);

// Allocation-free variant (no counterpart in the reference).  Identical to
// sh_paged_attention except that params->part_o / part_ml are ignored: the
// split-KV partials live in a fixed device array inside this library, so the
// call performs no device allocation of any kind.  It exists for callers that
// cannot allocate device memory where they run attention (a host runtime
// without its own device allocator, a fixed pre-reserved memory budget, or a
// latency path that must not pay cudaMalloc's implicit synchronisation).
//   * Limit: num_tokens * hq * nsplit * (head_dim + 2) floats must not exceed
//     sh_paged_attention_noalloc_capacity() (SH_ATTN_NOALLOC_MAX_FLOATS,
//     16 MiB of fp32); larger calls return SH_NOALLOC_ERR_TOO_LARGE.
//   * The first call on each device looks the array up with
//     cudaGetSymbolAddress (that device must be current); make it before any
//     CUDA-graph stream capture.
//   * All calls share the array: calls that overlap on the GPU race.
//   * Every GPU that loads the library holds the array until process exit.
#define SH_ATTN_NOALLOC_MAX_FLOATS (4ll * 1024 * 1024)
#define SH_NOALLOC_ERR_ARGS -101
#define SH_NOALLOC_ERR_TOO_LARGE -102
#define SH_NOALLOC_ERR_DEVICE -103
#define SH_NOALLOC_ERR_SYMBOL -104
int sh_paged_attention_noalloc(const AttnParams* params, int ntiles, int num_blocks, int head_dim, int max_rows,
                               cudaStream_t stream);
int64_t sh_paged_attention_noalloc_capacity(void);
#ifdef __cplusplus
}
#endif
