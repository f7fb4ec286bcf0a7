// Per-token MoE routing as block-level device functions, shared by the
// standalone router kernels (moe.cu) and the expert-parallel dispatch that
// routes its own tokens (ep_a2a.cu).  The first `nt` threads of the block do
// the strided work and the reductions run over their warps only, so a caller
// with a larger block gets bit-identical ids and weights to a router launched
// with `nt` threads.  Every thread of the block must call (block barriers).
//
//  * softmax: softmax over E logits, top-k, optional renormalisation
//    (Qwen3-Next router).
//  * sigmoid_grouped: sigmoid scores; selection on score + correction bias,
//    restricted to the top `topk_groups` of `n_groups` groups (group score =
//    sum of its two best biased scores); weights = unbiased scores of the
//    chosen experts, renormalised and scaled (DeepSeek-V3 / Kimi-K2 router).
#pragma once
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "moe.h"

namespace shk {
namespace route {

// Router block size for E experts (the standalone router's launch width).
__host__ __device__ inline int threads_for(int E) { return E >= 512 ? 512 : (E >= 256 ? 256 : 128); }

__device__ __forceinline__ float load_logit(const void* p, int64_t i, int is_bf16) {
  return is_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}

// Shared scratch of one routing call (besides the 2E floats of scores).
struct Scratch {
  float rv[32];
  int ri[32];
  float red[32];
  float gscore[64];
  int kept[64];
  float chosen_w[64];
  int chosen_i[64];
};

// Argmax over s[0:E) by the first nt threads (ties -> lowest index).
__device__ inline int block_argmax(const float* s, int E, int nt, Scratch& sc) {
  float best = -INFINITY;
  int idx = 0x7fffffff;
  if (static_cast<int>(threadIdx.x) < nt)
    for (int e = threadIdx.x; e < E; e += nt)
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
  if (lane == 0 && w < 32) {
    sc.rv[w] = best;
    sc.ri[w] = idx;
  }
  __syncthreads();
  best = sc.rv[0];
  idx = sc.ri[0];
  for (int i = 1; i < nt / 32; ++i)
    if (sc.rv[i] > best || (sc.rv[i] == best && sc.ri[i] < idx)) {
      best = sc.rv[i];
      idx = sc.ri[i];
    }
  return idx;
}

// ---------------------------------------------------------------- one warp per token
// The fast path: E a multiple of 32 up to 512, k <= 32, and either no group limit or 32 experts per group.
// Lane l holds experts l + 32 i in registers (i < E / 32), so a group is one register index across the warp.
// The selection is the block path's: same scores, ties to the lower expert index, the sigmoid weights and
// the renormalisation summed in the same order (bit-identical ids and sigmoid weights; the softmax
// denominator is summed in a different order).
constexpr int kWarpMaxPer = 16;

__host__ __device__ inline bool warp_path(const RouteParams& p) {
  return p.E % 32 == 0 && p.E <= 32 * kWarpMaxPer && p.k <= 32 && p.k >= 1 &&
         (!p.sigmoid_grouped || p.n_groups == 1 || p.E / p.n_groups == 32);
}

// Lane j < k returns chosen expert j and its final weight in (id, w); every lane of the warp must call.
__device__ inline void route_token_warp(const RouteParams& p, int64_t t, int& id, float& w) {
  const int lane = threadIdx.x & 31, n = p.E >> 5;
  float sel[kWarpMaxPer], val[kWarpMaxPer];
#pragma unroll
  for (int i = 0; i < kWarpMaxPer; ++i) {
    sel[i] = -INFINITY;
    val[i] = 0.f;
    if (i < n) sel[i] = load_logit(p.logits, t * p.E + lane + 32 * i, p.logits_bf16);
  }
  float denom = 1.f;
  if (!p.sigmoid_grouped) {
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kWarpMaxPer; ++i)
      if (i < n) mx = fmaxf(mx, sel[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kWarpMaxPer; ++i)
      if (i < n) {
        sel[i] = __expf(sel[i] - mx);
        val[i] = sel[i];
        sum += sel[i];
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    denom = sum;
  } else {
#pragma unroll
    for (int i = 0; i < kWarpMaxPer; ++i)
      if (i < n) {
        const float v = 1.f / (1.f + __expf(-sel[i]));
        val[i] = v;
        sel[i] = v + (p.bias ? p.bias[lane + 32 * i] : 0.f);
      }
    if (p.n_groups > 1) {  // group g = register index g: its score is the sum of its two best biased scores
      float gs[kWarpMaxPer];
#pragma unroll
      for (int g = 0; g < kWarpMaxPer; ++g) {
        gs[g] = -INFINITY;
        if (g >= n) continue;  // warp-uniform
        float b1 = sel[g], b2 = -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float o1 = __shfl_xor_sync(0xffffffffu, b1, o), o2 = __shfl_xor_sync(0xffffffffu, b2, o);
          const float hi = fmaxf(b1, o1);
          b2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
          b1 = hi;
        }
        gs[g] = b1 + b2;
      }
      uint32_t kept = 0;  // the top `topk_groups` groups, ties to the lower index (the same in every lane)
      for (int j = 0; j < p.topk_groups; ++j) {
        int best = -1;
        float bv = 0.f;
#pragma unroll
        for (int g = 0; g < kWarpMaxPer; ++g)
          if (g < n && !((kept >> g) & 1u) && (best < 0 || gs[g] > bv)) {
            best = g;
            bv = gs[g];
          }
        if (best >= 0) kept |= 1u << best;
      }
#pragma unroll
      for (int g = 0; g < kWarpMaxPer; ++g)
        if (g < n && !((kept >> g) & 1u)) sel[g] = -INFINITY;
    }
  }
  uint32_t taken = 0;
  id = 0;
  w = 0.f;
  for (int j = 0; j < p.k; ++j) {
    float bv = -INFINITY, bw = 0.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kWarpMaxPer; ++i) {
      const int e = lane + 32 * i;
      if (i < n && !((taken >> i) & 1u) && (sel[i] > bv || (sel[i] == bv && e < bi))) {
        bv = sel[i];
        bi = e;
        bw = val[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o), ow = __shfl_xor_sync(0xffffffffu, bw, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
        bw = ow;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == j) {
      id = bi;
      w = p.sigmoid_grouped ? bw : bw / denom;
    }
  }
  float tot = 0.f;
  for (int j = 0; j < p.k; ++j) tot += __shfl_sync(0xffffffffu, w, j);
  const bool norm = p.sigmoid_grouped ? (p.renorm && tot > 0.f) : p.renorm;
  w = (norm ? w / tot : w) * p.scale;
}

// Routes token t: on return (after the final barrier) sc.chosen_i[0:k] and sc.chosen_w[0:k] hold the
// experts and their final weights (renormalised and scaled).  s: 2E floats of shared memory.
__device__ inline void route_token(const RouteParams& p, int64_t t, int nt, float* s, Scratch& sc) {
  const int tid = threadIdx.x;
  if (warp_path(p)) {  // warp 0 routes; the block only waits for the result
    if (tid < 32) {
      int id;
      float w;
      route_token_warp(p, t, id, w);
      if (tid < p.k) {
        sc.chosen_i[tid] = id;
        sc.chosen_w[tid] = w;
      }
    }
    __syncthreads();
    return;
  }
  const bool act = tid < nt;
  if (!p.sigmoid_grouped) {
    float mx = -INFINITY;
    if (act)
      for (int e = tid; e < p.E; e += nt) {
        s[e] = load_logit(p.logits, t * p.E + e, p.logits_bf16);
        mx = fmaxf(mx, s[e]);
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0 && act) sc.red[tid >> 5] = mx;
    __syncthreads();
    mx = sc.red[0];
    for (int i = 1; i < nt / 32; ++i) mx = fmaxf(mx, sc.red[i]);
    __syncthreads();
    float sum = 0.f;
    if (act)
      for (int e = tid; e < p.E; e += nt) {
        s[e] = __expf(s[e] - mx);
        sum += s[e];
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((tid & 31) == 0 && act) sc.red[tid >> 5] = sum;
    __syncthreads();
    sum = 0.f;
    for (int i = 0; i < nt / 32; ++i) sum += sc.red[i];
    for (int j = 0; j < p.k; ++j) {
      const int e = block_argmax(s, p.E, nt, sc);
      if (tid == 0) {
        sc.chosen_i[j] = e;
        sc.chosen_w[j] = s[e] / sum;
        s[e] = -INFINITY;
      }
      __syncthreads();
    }
  } else {
    float* sb = s + p.E;
    if (act)
      for (int e = tid; e < p.E; e += nt) {
        const float x = load_logit(p.logits, t * p.E + e, p.logits_bf16);
        const float v = 1.f / (1.f + __expf(-x));
        s[e] = v;
        sb[e] = v + (p.bias ? p.bias[e] : 0.f);
      }
    __syncthreads();
    const int per = p.E / p.n_groups;
    if (p.n_groups > 1) {
      if (act)
        for (int gi = tid; gi < p.n_groups; gi += nt) {
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
          sc.gscore[gi] = b1 + (per > 1 ? b2 : 0.f);
        }
      __syncthreads();
      if (tid == 0) {  // keep the top `topk_groups` groups (ties -> lower index), mask the rest
        for (int gi = 0; gi < p.n_groups; ++gi) sc.kept[gi] = 0;
        for (int j = 0; j < p.topk_groups; ++j) {
          int best = -1;
          for (int gi = 0; gi < p.n_groups; ++gi)
            if (!sc.kept[gi] && (best < 0 || sc.gscore[gi] > sc.gscore[best])) best = gi;
          if (best >= 0) sc.kept[best] = 1;
        }
      }
      __syncthreads();
      if (act)
        for (int e = tid; e < p.E; e += nt)
          if (!sc.kept[e / per]) sb[e] = -INFINITY;
      __syncthreads();
    }
    for (int j = 0; j < p.k; ++j) {
      const int e = block_argmax(sb, p.E, nt, sc);
      if (tid == 0) {
        sc.chosen_i[j] = e;
        sc.chosen_w[j] = s[e];
        sb[e] = -INFINITY;
      }
      __syncthreads();
    }
  }
  if (tid == 0) {
    float tot = 0.f;
    for (int j = 0; j < p.k; ++j) tot += sc.chosen_w[j];
    const bool norm = p.sigmoid_grouped ? (p.renorm && tot > 0.f) : p.renorm;
    for (int j = 0; j < p.k; ++j) sc.chosen_w[j] = (norm ? sc.chosen_w[j] / tot : sc.chosen_w[j]) * p.scale;
  }
  __syncthreads();
}

}  // namespace route
}  // namespace shk
