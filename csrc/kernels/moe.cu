// Mixture-of-experts routing and token movement.
//
//  * route_softmax_topk: softmax over E router logits, top-k, optional
//    renormalisation of the k weights (Qwen3-Next router).
//  * route_sigmoid_grouped: sigmoid scores; selection on score + correction
//    bias, restricted to the top `topk_groups` of `n_groups` expert groups
//    (group score = sum of its two best biased scores); weights = unbiased
//    scores of the chosen experts, renormalised and scaled (DeepSeek-V3 /
//    Kimi-K2 router).
//  * align: counting sort of the (token, slot) pairs by expert, exclusive
//    offsets, and the device-side tile list (sorted row start, rows, expert
//    weight row offset) the grouped tcgen05 GEMM consumes -- no host sync.
//  * gather / combine: sorted activation rows in, weighted per-token sum out
//    (fixed slot order, so results do not depend on the sort order).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "moe.h"
#include "pdl.cuh"

namespace shk {
namespace moe {

__device__ __forceinline__ float load_f(const void* p, int64_t i, int is_bf16) {
  return is_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}

// Block argmax over s[0:E) (ties -> lowest index); returns the index.
__device__ int block_argmax(const float* s, int E, float* rv, int* ri) {
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    if (s[e] > best || (s[e] == best && e < idx)) {
      best = s[e];
      idx = e;
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) {
      best = ob;
      idx = oi;
    }
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) {
    rv[w] = best;
    ri[w] = idx;
  }
  __syncthreads();
  best = rv[0];
  idx = ri[0];
  for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i)
    if (rv[i] > best || (rv[i] == best && ri[i] < idx)) {
      best = rv[i];
      idx = ri[i];
    }
  return idx;
}

__global__ void route_softmax_kernel(RouteParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  extern __shared__ float s[];
  __shared__ float rv[32];
  __shared__ int ri[32];
  __shared__ float red[32];
  const int64_t t = blockIdx.x;
  float mx = -INFINITY;
  for (int e = threadIdx.x; e < p.E; e += blockDim.x) {
    s[e] = load_f(p.logits, t * p.E + e, p.logits_bf16);
    mx = fmaxf(mx, s[e]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i) mx = fmaxf(mx, red[i]);
  __syncthreads();
  float sum = 0.f;
  for (int e = threadIdx.x; e < p.E; e += blockDim.x) {
    s[e] = __expf(s[e] - mx);
    sum += s[e];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  sum = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) sum += red[i];
  __shared__ float chosen_w[64];
  __shared__ int chosen_i[64];
  for (int j = 0; j < p.k; ++j) {
    const int e = block_argmax(s, p.E, rv, ri);
    if (threadIdx.x == 0) {
      chosen_i[j] = e;
      chosen_w[j] = s[e] / sum;
      s[e] = -INFINITY;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int j = 0; j < p.k; ++j) tot += chosen_w[j];
    for (int j = 0; j < p.k; ++j) {
      p.ids[t * p.k + j] = chosen_i[j];
      p.weights[t * p.k + j] = (p.renorm ? chosen_w[j] / tot : chosen_w[j]) * p.scale;
    }
  }
}

__global__ void route_sigmoid_grouped_kernel(RouteParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  extern __shared__ float s[];  // [E] scores, [E] biased
  float* sb = s + p.E;
  __shared__ float rv[32];
  __shared__ int ri[32];
  __shared__ float gscore[64];
  __shared__ float chosen_w[64];
  __shared__ int chosen_i[64];
  const int64_t t = blockIdx.x;
  for (int e = threadIdx.x; e < p.E; e += blockDim.x) {
    const float x = load_f(p.logits, t * p.E + e, p.logits_bf16);
    const float sc = 1.f / (1.f + __expf(-x));
    s[e] = sc;
    sb[e] = sc + (p.bias ? p.bias[e] : 0.f);
  }
  __syncthreads();
  const int per = p.E / p.n_groups;
  if (p.n_groups > 1) {
    // Group score: sum of the two best biased scores in the group.
    for (int gi = threadIdx.x; gi < p.n_groups; gi += blockDim.x) {
      float b1 = -INFINITY, b2 = -INFINITY;
      for (int e = gi * per; e < (gi + 1) * per; ++e) {
        const float v = sb[e];
        if (v > b1) {
          b2 = b1;
          b1 = v;
        } else if (v > b2) {
          b2 = v;
        }
      }
      gscore[gi] = b1 + (per > 1 ? b2 : 0.f);
    }
    __syncthreads();
    __shared__ int kept[64];
    if (threadIdx.x == 0) {  // keep the top `topk_groups` groups (ties -> lower index), mask the rest
      for (int gi = 0; gi < p.n_groups; ++gi) kept[gi] = 0;
      for (int j = 0; j < p.topk_groups; ++j) {
        int best = -1;
        for (int gi = 0; gi < p.n_groups; ++gi)
          if (!kept[gi] && (best < 0 || gscore[gi] > gscore[best])) best = gi;
        if (best >= 0) kept[best] = 1;
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < p.E; e += blockDim.x)
      if (!kept[e / per]) sb[e] = -INFINITY;
    __syncthreads();
  }
  for (int j = 0; j < p.k; ++j) {
    const int e = block_argmax(sb, p.E, rv, ri);
    if (threadIdx.x == 0) {
      chosen_i[j] = e;
      chosen_w[j] = s[e];
      sb[e] = -INFINITY;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int j = 0; j < p.k; ++j) tot += chosen_w[j];
    for (int j = 0; j < p.k; ++j) {
      p.ids[t * p.k + j] = chosen_i[j];
      p.weights[t * p.k + j] = (p.renorm && tot > 0.f ? chosen_w[j] / tot : chosen_w[j]) * p.scale;
    }
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
  const int threads = p->E >= 512 ? 512 : (p->E >= 256 ? 256 : 128);
  if (p->sigmoid_grouped) {
    if (p->n_groups < 1 || p->E % p->n_groups || p->n_groups > 64) return -2;
    shk::launch(route_sigmoid_grouped_kernel, dim3(p->T), dim3(threads), 2 * p->E * sizeof(float), stream, *p);
  } else {
    shk::launch(route_softmax_kernel, dim3(p->T), dim3(threads), p->E * sizeof(float), stream, *p);
  }
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
