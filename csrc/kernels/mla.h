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
// NVFP4 latent cache row (Cl latent + R rope values), the row of vLLM's `nvfp4_ds_mla` cache: [0, Cl/2)
// e2m1 pairs (low nibble = even dim), [Cl/2, Cl/2 + R) the rope values as unscaled e4m3, then Cl/16 e4m3
// block scales, scale s stored at byte (Cl/64) * (s % 4) + s / 4 of that region; rows padded to 16 bytes
// (Cl 512, R 64: 352 bytes against 1152 in bf16).  Block scale sc = e4m3(max(amax16 / 6, 2^-9)), code =
// e2m1_rne(x * (1 / sc)); the value read back is code * sc, the rope value e4m3_rne_satfinite(x).
int sh_mla_fp4_row_bytes(int Cl, int R);
int sh_mla_cache_write_fp4(uint8_t* cache, const __nv_bfloat16* c, int64_t c_stride, const __nv_bfloat16* kpe,
                           int64_t kpe_stride, const int64_t* slots, int T, int Cl, int R, cudaStream_t stream);
// latent[slot[t]] = cat(c[t], kpe[t]) for slot[t] >= 0 (C = Cl + R).
int sh_mla_cache_write(__nv_bfloat16* latent, const __nv_bfloat16* c, int64_t c_stride, const __nv_bfloat16* kpe,
                       int64_t kpe_stride, const int64_t* slots, int T, int Cl, int R, cudaStream_t stream);
#ifdef __cplusplus
}
#endif

#if defined(__CUDACC__)
#include <cuda_fp16.h>
#include <cuda_fp8.h>
// Eight e4m3 bytes (value i in byte i) -> eight bf16 as four bf16x2 words, exact: every e4m3 value is an
// f16 normal and a bf16 value (hardware e4m3x2 -> f16x2 conversion, then f16 -> fp32 -> bf16).
__device__ __forceinline__ void e4m3x8_to_bf16(uint2 v, uint32_t* out) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w = i < 2 ? v.x : v.y;
    const __half2_raw hr =
        __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>((w >> (16 * (i & 1))) & 0xFFFFu), __NV_E4M3);
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
    const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
    out[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
}
#endif
