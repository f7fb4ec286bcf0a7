// Memory-bound fused kernels of the decoder layer.
//
//  * rms_norm / fused_add_rms_norm: one CTA per token row, vectorised 16-byte
//    loads, fp32 accumulation; the fused variant adds the residual in place
//    and normalises in the same pass (one read + two writes per element).
//  * rope_kv_write: rotates q and k of the QKV projection output in place
//    (NeoX rotate-half form) and scatters k, v into the paged cache
//    [num_blocks, kv_heads, block, head_dim] in one pass.
//  * silu_mul: SwiGLU activation over the fused gate|up projection.
//  * embedding: token gather.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "pdl.cuh"

namespace shk {

template <typename T>
__global__ void rms_norm_kernel(T* __restrict__ out, const T* __restrict__ x, const T* __restrict__ w, int hidden,
                                int64_t x_stride, int64_t out_stride, float eps) {
  shk::pdl_trigger();
  shk::pdl_wait();
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * x_stride;
  T* orow = out + row * out_stride;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float v = to_f(xr[i]);
    ss += v * v;
  }
  ss = block_sum(ss, scratch);
  const float inv = rsqrtf(ss / hidden + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) orow[i] = from_f<T>(to_f(xr[i]) * inv * to_f(w[i]));
}

// bf16, hidden % 8 == 0: 16-byte vectors, residual += x, x = norm(residual) * w.
__global__ void fused_add_rms_norm_bf16_kernel(__nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                                               const __nv_bfloat16* __restrict__ w, int hidden, float eps) {
  shk::pdl_trigger();
  shk::pdl_wait();
  __shared__ float scratch[32];
  extern __shared__ float4 row_cache[];  // hidden bf16 of the summed row
  const int64_t row = blockIdx.x;
  const int nvec = hidden / 8;
  float4* xv = reinterpret_cast<float4*>(x + row * hidden);
  float4* rv = reinterpret_cast<float4*>(residual + row * hidden);
  float ss = 0.f;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float4 a = xv[i], b = rv[i];
    __nv_bfloat162* ap = reinterpret_cast<__nv_bfloat162*>(&a);
    __nv_bfloat162* bp = reinterpret_cast<__nv_bfloat162*>(&b);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fa = __bfloat1622float2(ap[j]);
      const float2 fb = __bfloat1622float2(bp[j]);
      const float2 s = make_float2(fa.x + fb.x, fa.y + fb.y);
      bp[j] = __float22bfloat162_rn(s);
      const float2 r = __bfloat1622float2(bp[j]);
      ss += r.x * r.x + r.y * r.y;
    }
    rv[i] = b;
    row_cache[i] = b;
  }
  ss = block_sum(ss, scratch);
  const float inv = rsqrtf(ss / hidden + eps);
  const float4* wv = reinterpret_cast<const float4*>(w);
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float4 b = row_cache[i], ww = wv[i], o;
    const __nv_bfloat162* bp = reinterpret_cast<const __nv_bfloat162*>(&b);
    const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&ww);
    __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fb = __bfloat1622float2(bp[j]);
      const float2 fw = __bfloat1622float2(wp[j]);
      op[j] = __float22bfloat162_rn(make_float2(fb.x * inv * fw.x, fb.y * inv * fw.y));
    }
    xv[i] = o;
  }
}

template <typename T>
__global__ void fused_add_rms_norm_kernel(T* __restrict__ x, T* __restrict__ residual, const T* __restrict__ w,
                                          int hidden, float eps) {
  shk::pdl_trigger();
  shk::pdl_wait();
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  T* xr = x + row * hidden;
  T* rr = residual + row * hidden;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const T s = from_f<T>(to_f(xr[i]) + to_f(rr[i]));
    rr[i] = s;
    const float f = to_f(s);
    ss += f * f;
  }
  ss = block_sum(ss, scratch);
  const float inv = rsqrtf(ss / hidden + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) xr[i] = from_f<T>(to_f(rr[i]) * inv * to_f(w[i]));
}

// qkv: [T, (Hq + 2 Hk) * D] (row stride qkv_stride).  cos_sin: [max_pos, rot] with
// cos in [:rot/2] and sin in [rot/2:].  Rotary applies to the first `rot`
// dims of each head (rot <= D, partial rotary), NeoX rotate-half pairing.
template <typename T>
__global__ void rope_kv_write_kernel(T* __restrict__ qkv, int64_t qkv_stride, const int64_t* __restrict__ positions,
                                     const float* __restrict__ cos_sin, T* __restrict__ k_cache,
                                     T* __restrict__ v_cache, const int64_t* __restrict__ slot_mapping, int hq, int hk,
                                     int d, int rot, int block_size) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int64_t tok = blockIdx.x;
  T* row = qkv + tok * qkv_stride;
  const int64_t pos = positions[tok];
  const float* cs = cos_sin + pos * rot;
  const int half = rot / 2;
  const int nheads = hq + hk;
  // Rotate q heads and k heads in place.
  for (int idx = threadIdx.x; idx < nheads * half; idx += blockDim.x) {
    const int h = idx / half, i = idx % half;
    T* hp = row + h * d;
    const float c = cs[i], s = cs[half + i];
    const float x1 = to_f(hp[i]), x2 = to_f(hp[i + half]);
    hp[i] = from_f<T>(x1 * c - x2 * s);
    hp[i + half] = from_f<T>(x2 * c + x1 * s);
  }
  __syncthreads();
  const int64_t slot = slot_mapping[tok];
  if (slot < 0) return;  // padded token: nothing cached
  const int64_t blk = slot / block_size, off = slot % block_size;
  const T* kp = row + hq * d;
  const T* vp = row + (hq + hk) * d;
  for (int idx = threadIdx.x; idx < hk * d; idx += blockDim.x) {
    const int h = idx / d, i = idx % d;
    const int64_t dst = ((blk * hk + h) * block_size + off) * d + i;
    k_cache[dst] = kp[idx];
    v_cache[dst] = vp[idx];
  }
}

template <typename T>
__global__ void silu_mul_kernel(T* __restrict__ out, const T* __restrict__ x, int f) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int64_t row = blockIdx.x;
  const T* g = x + row * 2 * f;
  const T* u = g + f;
  T* o = out + row * f;
  for (int i = threadIdx.x; i < f; i += blockDim.x) {
    const float gv = to_f(g[i]);
    o[i] = from_f<T>(gv / (1.f + __expf(-gv)) * to_f(u[i]));
  }
}

__global__ void silu_mul_bf16_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x, int f) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int64_t row = blockIdx.x;
  const float4* g = reinterpret_cast<const float4*>(x + row * 2 * f);
  const float4* u = reinterpret_cast<const float4*>(x + row * 2 * f + f);
  float4* o = reinterpret_cast<float4*>(out + row * f);
  for (int i = threadIdx.x; i < f / 8; i += blockDim.x) {
    float4 gv = g[i], uv = u[i], ov;
    const __nv_bfloat162* gp = reinterpret_cast<const __nv_bfloat162*>(&gv);
    const __nv_bfloat162* up = reinterpret_cast<const __nv_bfloat162*>(&uv);
    __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 a = __bfloat1622float2(gp[j]);
      const float2 b = __bfloat1622float2(up[j]);
      op[j] = __float22bfloat162_rn(make_float2(a.x / (1.f + __expf(-a.x)) * b.x, a.y / (1.f + __expf(-a.y)) * b.y));
    }
    o[i] = ov;
  }
}

template <typename T>
__global__ void embedding_kernel(T* __restrict__ out, const int64_t* __restrict__ ids, const T* __restrict__ table,
                                 int hidden, int64_t vocab) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int64_t row = blockIdx.x;
  int64_t id = ids[row];
  if (id < 0 || id >= vocab) id = 0;  // out-of-range ids read row 0, never out of bounds
  const T* src = table + id * hidden;
  T* dst = out + row * hidden;
  if ((hidden * sizeof(T)) % 16 == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    for (int i = threadIdx.x; i < hidden * (int)sizeof(T) / 16; i += blockDim.x) d4[i] = s4[i];
  } else {
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = src[i];
  }
}

}  // namespace shk

using namespace shk;

#define SH_DISPATCH(dtype, ...)                                                  \
  if (dtype == at::kBFloat16) {                                                  \
    using scalar = __nv_bfloat16;                                                \
    __VA_ARGS__                                                                  \
  } else if (dtype == at::kHalf) {                                               \
    using scalar = __half;                                                       \
    __VA_ARGS__                                                                  \
  } else if (dtype == at::kFloat) {                                              \
    using scalar = float;                                                        \
    __VA_ARGS__                                                                  \
  } else {                                                                       \
    TORCH_CHECK(false, "unsupported dtype ", dtype);                             \
  }

static int threads_for(int n) {
  int t = 32;
  while (t < n && t < 1024) t <<= 1;
  return t;
}

void rms_norm(torch::Tensor out, torch::Tensor x, torch::Tensor w, double eps) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1, "rms_norm: bad x/out");
  TORCH_CHECK(w.is_contiguous() && w.numel() == x.size(1), "rms_norm: bad weight");
  const int hidden = x.size(1);
  const int64_t rows = x.size(0);
  if (rows == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  SH_DISPATCH(x.scalar_type(), {
    shk::launch(rms_norm_kernel<scalar>, dim3(rows), dim3(threads_for(std::min(hidden / 4, 1024))), 0, stream, 
        (scalar*)out.data_ptr(), (const scalar*)x.data_ptr(), (const scalar*)w.data_ptr(), hidden, x.stride(0),
        out.stride(0), (float)eps);
  });
  SH_CUDA_CHECK(cudaGetLastError());
}

void fused_add_rms_norm(torch::Tensor x, torch::Tensor residual, torch::Tensor w, double eps) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && residual.is_contiguous() && x.sizes() == residual.sizes(),
              "fused_add_rms_norm: bad tensors");
  const int hidden = x.size(-1);
  const int64_t rows = x.numel() / hidden;
  if (rows == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kBFloat16 && hidden % 8 == 0) {
    const int threads = threads_for(std::min(hidden / 8, 1024));
    shk::launch(fused_add_rms_norm_bf16_kernel, dim3(rows), dim3(threads), hidden * 2, stream, 
        (__nv_bfloat16*)x.data_ptr(), (__nv_bfloat16*)residual.data_ptr(), (const __nv_bfloat16*)w.data_ptr(), hidden,
        (float)eps);
  } else {
    SH_DISPATCH(x.scalar_type(), {
      shk::launch(fused_add_rms_norm_kernel<scalar>, dim3(rows), dim3(threads_for(std::min(hidden, 1024))), 0, stream, 
          (scalar*)x.data_ptr(), (scalar*)residual.data_ptr(), (const scalar*)w.data_ptr(), hidden, (float)eps);
    });
  }
  SH_CUDA_CHECK(cudaGetLastError());
}

void rope_kv_write(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin, torch::Tensor k_cache,
                   torch::Tensor v_cache, torch::Tensor slot_mapping, int64_t hq, int64_t hk, int64_t d, int64_t rot) {
  TORCH_CHECK(qkv.is_cuda() && qkv.dim() == 2 && qkv.stride(1) == 1, "rope_kv_write: qkv must be [T, width]");
  TORCH_CHECK(qkv.size(1) >= (hq + 2 * hk) * d, "rope_kv_write: qkv too narrow");
  TORCH_CHECK(positions.scalar_type() == at::kLong && slot_mapping.scalar_type() == at::kLong, "int64 indices");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == rot, "cos_sin must be f32 [pos, rot]");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(1) == hk && k_cache.size(3) == d, "cache [blocks, hk, bs, d]");
  const int64_t t = qkv.size(0);
  if (t == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  SH_DISPATCH(qkv.scalar_type(), {
    shk::launch(rope_kv_write_kernel<scalar>, dim3(t), dim3(256), 0, stream, 
        (scalar*)qkv.data_ptr(), qkv.stride(0), positions.data_ptr<int64_t>(), cos_sin.data_ptr<float>(),
        (scalar*)k_cache.data_ptr(), (scalar*)v_cache.data_ptr(), slot_mapping.data_ptr<int64_t>(), hq, hk, d, rot,
        k_cache.size(2));
  });
  SH_CUDA_CHECK(cudaGetLastError());
}

void silu_mul(torch::Tensor out, torch::Tensor x) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && out.is_contiguous(), "silu_mul: contiguous tensors");
  const int f = out.size(-1);
  TORCH_CHECK(x.size(-1) == 2 * f, "silu_mul: x must be [.., 2F]");
  const int64_t rows = out.numel() / f;
  if (rows == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kBFloat16 && f % 8 == 0) {
    shk::launch(silu_mul_bf16_kernel, dim3(rows), dim3(threads_for(std::min(f / 8, 1024))), 0, stream, 
        (__nv_bfloat16*)out.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), f);
  } else {
    SH_DISPATCH(x.scalar_type(), {
      shk::launch(silu_mul_kernel<scalar>, dim3(rows), dim3(threads_for(std::min(f, 1024))), 0, stream, (scalar*)out.data_ptr(),
                                                                                   (const scalar*)x.data_ptr(), f);
    });
  }
  SH_CUDA_CHECK(cudaGetLastError());
}

void embedding(torch::Tensor out, torch::Tensor ids, torch::Tensor table) {
  TORCH_CHECK(table.is_contiguous() && out.is_contiguous() && ids.scalar_type() == at::kLong && ids.is_contiguous(),
              "embedding: contiguous int64 ids, table and out");
  const int64_t rows = ids.numel();
  if (rows == 0) return;
  const int hidden = table.size(1);
  auto stream = at::cuda::getCurrentCUDAStream();
  SH_DISPATCH(table.scalar_type(), {
    shk::launch(embedding_kernel<scalar>, dim3(rows), dim3(128), 0, stream, (scalar*)out.data_ptr(), ids.data_ptr<int64_t>(),
                                                       (const scalar*)table.data_ptr(), hidden, table.size(0));
  });
  SH_CUDA_CHECK(cudaGetLastError());
}
