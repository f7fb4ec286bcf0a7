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
#ifdef __cplusplus
}
#endif
