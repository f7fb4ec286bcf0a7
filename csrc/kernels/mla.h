// C ABI of the MLA (multi-head latent attention) decode kernels and the DSA indexer.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

struct MlaParams {
  const __nv_bfloat16* q;       // [T, H, C] absorbed queries: [q_nope W_UK | rotated q_pe]
  const __nv_bfloat16* latent;  // paged cache [num_blocks, 64, C]: [normalised c_kv | rotated k_pe]
  const uint8_t* latent_fp4;    // or the NVFP4 cache [num_blocks, 64, row_bytes] (see sh_mla_fp4_row_bytes)
  const int32_t* block_tables;  // [B, bt_stride]
  int64_t bt_stride;
  const int64_t* seq_lens;      // [B] keys of the request including its new tokens
  const int64_t* q_start;       // [B+1] query start offsets (a token's request is found by binary search)
  int B;
  const int32_t* topk;          // [T, topk_k] absolute key positions (-1 unused) or nullptr (dense causal)
  int topk_k;
  __nv_bfloat16* out;           // [T, H, V] (nsplit == 1)
  float* part_o;                // [T, H, nsplit, V]  (nsplit > 1)
  float* part_ml;               // [T, H, nsplit, 2]  (log2-domain max, sum)
  int* err;
  int T, H, nsplit;
  float scale_log2;             // softmax scale * log2(e)
  int impl;                     // 0: tcgen05 kernel where it applies, 1: the mma.sync kernel only
  unsigned long long* stamps;   // optional per-CTA cycle counters of the tcgen05 kernel ([grid][8]; profiling)
};


#ifdef __cplusplus
extern "C" {
#endif
// C % 64 == 0 and V % 64 == 0 (V <= C); supported (C, V): (576, 512), (128, 64).
// Uses the tcgen05 kernel (mla_tc.cu) for C = 576, V = 512, H % 128 == 0 and a bf16 cache unless impl == 1.
int sh_mla_decode(const MlaParams* p, int C, int V, cudaStream_t stream);
// The tcgen05 kernel alone (no split merge): -2 when it does not apply to p.
int sh_mla_decode_tc(const MlaParams* p, cudaStream_t stream);
// NVFP4 latent cache row (Cl latent + R rope values): Cl/2 bytes of e2m1 pairs (low nibble first), Cl/16
// e4m3 block scales at byte Cl/2, the R rope values in bf16 at the next 16-byte boundary; rows padded
// to 16 bytes (Cl 512, R 64: 416 bytes against 1152 in bf16).  Block scale s = e4m3(amax16 / 6),
// code = e2m1_rne(x / s); the value read back is code * s.
int sh_mla_fp4_row_bytes(int Cl, int R);
int sh_mla_cache_write_fp4(uint8_t* cache, const __nv_bfloat16* c, int64_t c_stride, const __nv_bfloat16* kpe,
                           int64_t kpe_stride, const int64_t* slots, int T, int Cl, int R, cudaStream_t stream);
// latent[slot[t]] = cat(c[t], kpe[t]) for slot[t] >= 0 (C = Cl + R).
int sh_mla_cache_write(__nv_bfloat16* latent, const __nv_bfloat16* c, int64_t c_stride, const __nv_bfloat16* kpe,
                       int64_t kpe_stride, const int64_t* slots, int T, int Cl, int R, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
