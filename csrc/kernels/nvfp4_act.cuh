// NVFP4 activation quantisation building blocks shared by the activation
// quantiser (gemm_fp4mma.cu) and the quantising expert-parallel dispatch
// (ep_a2a.cu): both produce bit-identical codes and scales for a row.
//   g = 2688 / amax(|row|) (1 for a zero row), or a static g;
//   per 16 values: s = e4m3(min(amax16 * g / 6, 448)), code = e2m1(x * g / s).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace shk {
namespace nvq {

// Eight values -> eight e2m1 codes (round to nearest even, saturating at 6; the
// sign bit is kept for negative values that round to zero), element 2i in the
// low nibble of byte i.
__device__ __forceinline__ uint32_t e2m1x8(const float* v) {
  uint32_t out;
  asm("{\n .reg .b8 b0, b1, b2, b3;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n"
      " mov.b32 %0, {b0, b1, b2, b3};\n}"
      : "=r"(out)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return out;
}

__device__ __forceinline__ void load16(const __nv_bfloat16* p, float* v) {
  const uint4 u0 = *reinterpret_cast<const uint4*>(p);
  const uint4 u1 = *reinterpret_cast<const uint4*>(p + 8);
  const __nv_bfloat162* h0 = reinterpret_cast<const __nv_bfloat162*>(&u0);
  const __nv_bfloat162* h1 = reinterpret_cast<const __nv_bfloat162*>(&u1);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 a = __bfloat1622float2(h0[j]);
    const float2 c = __bfloat1622float2(h1[j]);
    v[2 * j] = a.x;
    v[2 * j + 1] = a.y;
    v[8 + 2 * j] = c.x;
    v[8 + 2 * j + 1] = c.y;
  }
}


// Row multiplier from the row's absolute maximum.
__device__ __forceinline__ float row_g(float amax) { return amax > 0.f ? __fdiv_rn(2688.f, amax) : 1.f; }

// One 16-value block: writes the eight code bytes to `q` and returns the e4m3 scale byte.
__device__ __forceinline__ uint8_t quant16(float* v, float g, float g6, uint8_t* q) {
  float am = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) am = fmaxf(am, fabsf(v[j]));
  const __nv_fp8_e4m3 s(fminf(am * g6, 448.f));  // round to nearest even, saturating
  const float sfv = static_cast<float>(s);
  const float inv = sfv > 0.f ? __fdiv_rn(g, sfv) : 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] *= inv;
  *reinterpret_cast<uint2*>(q) = make_uint2(e2m1x8(v), e2m1x8(v + 8));
  return s.__x;
}

}  // namespace nvq
}  // namespace shk
