// DeepSeek-V3.2 lightning indexer (DSA) on sm_100a: fp8 paged index-key cache,
// tcgen05 scoring over key tiles shared by all query rows of a request, and a
// per-token top-k select.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// Index-key cache page (64 keys): 64 x 128 e4m3 key bytes, then 64 f32 per-key
// scales -> 8448 bytes (132 B per key).  A key reads back as e4m3 * scale.
#define SH_DSA_PAGE_KEYS 64
#define SH_DSA_DIM 128
#define SH_DSA_PAGE_BYTES (SH_DSA_PAGE_KEYS * (SH_DSA_DIM + 4))

struct DsaIndexParams {
  const uint8_t* q8;           // [T, IH, 128] e4m3 queries (per-row scale folded into wq)
  const float* wq;             // [T, IH] head weight x query scale
  const uint8_t* kcache;       // [num_pages, 8448] pages
  int num_pages;
  const int32_t* block_tables;  // [B, bt_stride] page ids
  int64_t bt_stride;
  const int64_t* seq_lens;     // [B] keys in the cache per request (queries included)
  const int64_t* q_start;      // [B + 1] first query row of each request
  int B, T, IH, K;
  float* logits;               // [T, ld] scratch; row t holds positions [0, pos_t]
  int64_t ld;
  int32_t* topk;               // [T, K] selected positions, ascending, -1 padded
  int* err;                    // wait timeouts: 400 + phase
  int grid;                    // persistent scoring CTAs (<= SMs)
};

#ifdef __cplusplus
extern "C" {
#endif
// cache[slot[t] / 64] row slot[t] % 64 <- e4m3(k[t] / s), s = amax(|k[t]|) / 448 (1 when k[t] == 0).
int sh_dsa_cache_write(uint8_t* cache, const __nv_bfloat16* k, int64_t k_stride, const int64_t* slots, int T,
                       cudaStream_t stream);
// q8[r] = e4m3(q[r] / s_r), wq[r] = w[r] * s_r for the T * IH rows of 128 values, s_r = amax / 448.
int sh_dsa_quant_q(uint8_t* q8, float* wq, const __nv_bfloat16* q, const float* w, int rows, cudaStream_t stream);
// logits[t, p] = ks[p] * sum_h relu(q8[t, h] . k8[p]) * wq[t, h] for p <= pos_t, then the top K per token.
// IH in {16, 64}.
int sh_dsa_index(const DsaIndexParams* p, cudaStream_t stream);
// Scoring only (the logits rows), for benchmarks and tests.
int sh_dsa_score(const DsaIndexParams* p, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
