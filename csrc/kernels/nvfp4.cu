// NVFP4 (ModelOpt layout) weight quantisation and dequantisation.
//
// Layout (the checkpoint format the reference's quantiser writes, reference:
// suffix_hybrid/tools/quantize_nvfp4.py): `weight` uint8 [N, K/2], two e2m1
// codes per byte, low nibble = even column; `weight_scale` e4m3 [N, K/16], one
// scale per 16-element block; `weight_scale_2` fp32 global scale.  Value =
// e2m1(code) * e4m3(block scale) * global.  e2m1 magnitudes: 0, 0.5, 1, 1.5,
// 2, 3, 4, 6; bit 3 is the sign.
//
// quantize: global = amax(W) / (6 * 448); block scale = e4m3(block_amax / 6 /
// global); code = nearest e2m1 to w / (scale * global) (ties to the even
// code).  One thread per 16-element block, vectorised I/O.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include "pdl.cuh"

namespace shk {
namespace fp4 {

__device__ __constant__ float kE2M1[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};

__device__ __forceinline__ float e4m3_to_f(uint8_t b) {
  __nv_fp8_e4m3 v;
  v.__x = b;
  return static_cast<float>(v);
}
__device__ __forceinline__ uint8_t f_to_e4m3(float f) {
  __nv_fp8_e4m3 v(f);  // round-to-nearest-even, saturating
  return v.__x;
}

__device__ __forceinline__ uint8_t e2m1_code(float x) {
  const float a = fabsf(x);
  // Nearest magnitude; a value exactly between two goes to the even code
  // (round half to even on the code grid, as the ModelOpt / vLLM quantiser).
  uint8_t c = a <= 0.25f ? 0 : a < 0.75f ? 1 : a <= 1.25f ? 2 : a < 1.75f ? 3 : a <= 2.5f ? 4 : a < 3.5f ? 5 : a <= 5.f ? 6 : 7;
  return x < 0.f ? static_cast<uint8_t>(c | 8) : c;  // negative values keep the sign bit (-0 included)
}

__global__ void dequant_kernel(__nv_bfloat16* __restrict__ out, const uint8_t* __restrict__ packed,
                               const uint8_t* __restrict__ scales, const float* __restrict__ global, int64_t N, int K) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int64_t blocks_per_row = K / 16;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= N * blocks_per_row) return;
  const int64_t row = i / blocks_per_row, blk = i % blocks_per_row;
  const float s = e4m3_to_f(scales[i]) * global[0];
  const uint2 q = *reinterpret_cast<const uint2*>(packed + row * (K / 2) + blk * 8);
  const uint8_t* b = reinterpret_cast<const uint8_t*>(&q);
  uint4 o[2];
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(o);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint8_t lo = b[j] & 15, hi = b[j] >> 4;
    const float vl = (lo & 8 ? -1.f : 1.f) * kE2M1[lo & 7] * s;
    const float vh = (hi & 8 ? -1.f : 1.f) * kE2M1[hi & 7] * s;
    h[j] = __floats2bfloat162_rn(vl, vh);
  }
  uint4* dst = reinterpret_cast<uint4*>(out + row * K + blk * 16);
  dst[0] = o[0];
  dst[1] = o[1];
}

__global__ void quant_kernel(uint8_t* __restrict__ packed, uint8_t* __restrict__ scales,
                             const __nv_bfloat16* __restrict__ w, const float* __restrict__ global, int64_t N, int K) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int64_t blocks_per_row = K / 16;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= N * blocks_per_row) return;
  const int64_t row = i / blocks_per_row, blk = i % blocks_per_row;
  const __nv_bfloat16* src = w + row * K + blk * 16;
  float v[16];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    v[j] = __bfloat162float(src[j]);
    amax = fmaxf(amax, fabsf(v[j]));
  }
  // IEEE round-to-nearest divisions (not the fast-math approximations): values
  // that land exactly on a rounding midpoint are common with bf16 inputs, and
  // the tie rule only holds with exact quotients.
  const float g = global[0];
  const uint8_t sc = f_to_e4m3(g > 0.f ? __fdiv_rn(__fdiv_rn(amax, 6.f), g) : 0.f);
  scales[i] = sc;
  const float s = e4m3_to_f(sc) * g;
  const float d = s > 0.f ? s : 1.f;
  uint8_t out[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    out[j] = e2m1_code(__fdiv_rn(v[2 * j], d)) | (e2m1_code(__fdiv_rn(v[2 * j + 1], d)) << 4);
  *reinterpret_cast<uint2*>(packed + row * (K / 2) + blk * 8) = *reinterpret_cast<const uint2*>(out);
}

}  // namespace fp4
}  // namespace shk

extern "C" int sh_nvfp4_dequant(__nv_bfloat16* out, const uint8_t* packed, const uint8_t* scales, const float* global,
                                int64_t N, int K, cudaStream_t stream) {
  if (K % 16) return -1;
  const int64_t n = N * (K / 16);
  if (n == 0) return 0;
  shk::launch(shk::fp4::dequant_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, stream, out, packed, scales, global, N,
                                                                                         K);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_nvfp4_quant(uint8_t* packed, uint8_t* scales, const __nv_bfloat16* w, const float* global, int64_t N,
                              int K, cudaStream_t stream) {
  if (K % 16) return -1;
  const int64_t n = N * (K / 16);
  if (n == 0) return 0;
  shk::launch(shk::fp4::quant_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, stream, packed, scales, w, global, N, K);
  return static_cast<int>(cudaGetLastError());
}
