// Mixture-of-experts routing and token movement.
//
//  * route: one token per block; softmax top-k (Qwen3-Next) or sigmoid
//    group-limited (DeepSeek-V3 / Kimi-K2) selection, shared with the
//    expert-parallel dispatch through moe_route.cuh.
//  * align: counting sort of the (token, slot) pairs by expert, exclusive
//    offsets, and the device-side tile list (sorted row start, rows, expert
//    weight row offset) the grouped tcgen05 GEMM consumes -- no host sync.
//  * gather / combine: sorted activation rows in, weighted per-token sum out
//    (fixed slot order, so results do not depend on the sort order).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "moe.h"
#include "moe_route.cuh"
#include "pdl.cuh"

namespace shk {
namespace moe {

// One token per block; the selection itself is shk::route::route_token
// (moe_route.cuh), which the expert-parallel dispatch also runs per token.
__global__ void route_kernel(RouteParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  extern __shared__ float s[];  // [E] scores (softmax) or [E] scores + [E] biased (sigmoid_grouped)
  __shared__ shk::route::Scratch sc;
  const int64_t t = blockIdx.x;
  shk::route::route_token(p, t, blockDim.x, s, sc);
  if (threadIdx.x < p.k) {
    p.ids[t * p.k + threadIdx.x] = sc.chosen_i[threadIdx.x];
    p.weights[t * p.k + threadIdx.x] = sc.chosen_w[threadIdx.x];
  }
}

// Eight tokens per block, one warp each (shk::route::warp_path geometries).
__global__ void __launch_bounds__(256) route_warp_kernel(RouteParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int64_t t = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= p.T) return;  // warp-uniform
  int id;
  float w;
  shk::route::route_token_warp(p, t, id, w);
  const int lane = threadIdx.x & 31;
  if (lane < p.k) {
    p.ids[t * p.k + lane] = id;
    p.weights[t * p.k + lane] = w;
  }
}

// Single CTA: counting sort by expert + tile list.
__global__ void align_kernel(AlignParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  extern __shared__ int cnt[];  // [E] counts, then [E+1] offsets, [E] tile offsets
  int* off = cnt + p.E;
  int* toff = off + p.E + 1;
  for (int e = threadIdx.x; e < p.E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  const int pairs = p.T * p.k;
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int e = p.ids[i];
    p.rank[i] = (e >= 0 && e < p.E) ? atomicAdd(&cnt[e], 1) : -1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0, tacc = 0;
    for (int e = 0; e < p.E; ++e) {
      off[e] = acc;
      toff[e] = tacc;
      acc += cnt[e];
      tacc += (cnt[e] + p.bn - 1) / p.bn;
    }
    off[p.E] = acc;
    *p.num_groups = tacc < p.max_groups ? tacc : p.max_groups;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < p.E; e += blockDim.x) {
    p.offsets[e] = off[e];
    int ti = toff[e];
    for (int m0 = 0; m0 < cnt[e] && ti < p.max_groups; m0 += p.bn, ++ti)
      p.groups[ti] = make_int4(off[e] + m0, min(p.bn, cnt[e] - m0), e * p.rows_per_expert, e);
  }
  if (threadIdx.x == 0) p.offsets[p.E] = off[p.E];
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int e = p.ids[i];
    if (e < 0 || e >= p.E) {
      p.sorted_pos[i] = -1;
      continue;
    }
    const int pos = off[e] + p.rank[i];
    p.sorted_pos[i] = pos;
    p.sorted_token[pos] = i / p.k;
  }
}

__global__ void gather_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x,
                              const int32_t* __restrict__ sorted_token, const int* __restrict__ total, int H) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int row = blockIdx.x;
  if (row >= *total) return;
  const int t = sorted_token[row];
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t) * H);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// out[t] (+)= sum_j w[t, j] * y[sorted_pos[t*k + j]] in slot order; fp32 accumulate.
__global__ void combine_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ y,
                               const int32_t* __restrict__ sorted_pos, const float* __restrict__ w, int k, int H,
                               int accumulate) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int64_t t = blockIdx.x;
  for (int i = threadIdx.x; i < H / 2; i += blockDim.x) {
    float2 acc = accumulate ? __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(out + t * H)[i])
                            : make_float2(0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      const int pos = sorted_pos[t * k + j];
      if (pos < 0) continue;
      const float wj = w[t * k + j];
      const float2 v = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(y + static_cast<int64_t>(pos) * H)[i]);
      acc.x += wj * v.x;
      acc.y += wj * v.y;
    }
    reinterpret_cast<__nv_bfloat162*>(out + t * H)[i] = __floats2bfloat162_rn(acc.x, acc.y);
  }
}

}  // namespace moe
}  // namespace shk

using namespace shk::moe;

extern "C" int sh_moe_route(const RouteParams* p, cudaStream_t stream) {
  if (p->T <= 0) return 0;
  if (p->k > 64 || p->k < 1 || p->E < p->k) return -1;
  const int threads = shk::route::threads_for(p->E);
  if (p->sigmoid_grouped && (p->n_groups < 1 || p->E % p->n_groups || p->n_groups > 64)) return -2;
  if (shk::route::warp_path(*p)) {
    shk::launch(route_warp_kernel, dim3((p->T + 7) / 8), dim3(256), 0, stream, *p);
    return static_cast<int>(cudaGetLastError());
  }
  const size_t smem = (p->sigmoid_grouped ? 2 : 1) * p->E * sizeof(float);
  shk::launch(route_kernel, dim3(p->T), dim3(threads), smem, stream, *p);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_moe_align(const AlignParams* p, cudaStream_t stream) {
  if (p->T <= 0) return 0;
  const int smem = (3 * p->E + 1) * sizeof(int);
  if (smem > 200 * 1024) return -1;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(align_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  shk::launch(align_kernel, dim3(1), dim3(1024), smem, stream, *p);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_moe_gather(__nv_bfloat16* out, const __nv_bfloat16* x, const int32_t* sorted_token,
                             const int* total, int max_rows, int H, cudaStream_t stream) {
  if (max_rows <= 0) return 0;
  if (H % 8) return -1;
  shk::launch(gather_kernel, dim3(max_rows), dim3(128), 0, stream, out, x, sorted_token, total, H);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_moe_combine(__nv_bfloat16* out, const __nv_bfloat16* y, const int32_t* sorted_pos, const float* w,
                              int T, int k, int H, int accumulate, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (H % 2) return -1;
  shk::launch(combine_kernel, dim3(T), dim3(256), 0, stream, out, y, sorted_pos, w, k, H, accumulate);
  return static_cast<int>(cudaGetLastError());
}
