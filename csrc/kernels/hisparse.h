// C ABI of the host KV tier (HiSparse): device hot rows over a latent cache in mapped host memory.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

struct HsParams {
  const int32_t* topk;          // [T, K] absolute key positions of every query token (-1: none)
  int32_t* topk_out;            // [T, K] the same keys as hot-row indices of the request (-1: none)
  const int64_t* q_start;       // [B+1] query start offsets
  const int64_t* seq_lens;      // [B] keys of the request including its new tokens
  const int64_t* state_slots;   // [B] request slot: owner of H hot rows and of one residency map
  const int64_t* positions;     // [T] positions the step writes
  const int64_t* slot_mapping;  // [T] cache slots the step writes (-1: not written)
  const int32_t* block_tables;  // [B, bt_stride] blocks of the host-resident cache (64 rows each)
  int64_t bt_stride;
  const uint8_t* cold;          // host-resident rows [blocks * 64, row_bytes] (device-mapped pointer)
  uint8_t* hot;                 // device rows [slots * H, row_bytes]
  int32_t* pos2slot;            // [slots, P] hot row of a position (-1: not resident)
  int32_t* slot2pos;            // [slots, H] position a hot row holds (-1: free)
  int32_t* stamp;               // [slots, H] tick of the row's last use
  int32_t* clock;               // [slots] tick of the slot's last resolve
  int32_t* hot_bt;              // [B, H / 64] out: the request's hot block-table row
  int64_t* hot_seq;             // [B] out: a length that keeps every hot index causal (H + query tokens)
  int* err;                     // 601: more distinct keys than hot rows (the excess keys were dropped)
  int64_t* stats;               // [2] optional: += hits, += rows fetched from host memory
  int B, K, H, P, row_bytes;
};

#ifdef __cplusplus
extern "C" {
#endif
// H % 64 == 0, H <= 16384, row_bytes % 16 == 0.  One CTA of 1024 threads per request.
int sh_hisparse_resolve(const HsParams* p, cudaStream_t stream);
// Clears the residency of `n` request slots (before a slot is reused by a newly prefilled request).
int sh_hisparse_reset(int32_t* pos2slot, int32_t* slot2pos, int32_t* stamp, int32_t* clock, const int64_t* slots,
                      int n, int layers, int num_slots, int H, int P, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
