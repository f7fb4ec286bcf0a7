// Gated DeltaNet (Qwen3-Next linear attention) kernels with deferred commit.
//
// Speculative verify runs a window of W = k+1 tokens per request but only the
// first (accepted + 1) of them become history.  Instead of materialising W
// recurrent states, the window kernels leave the committed state untouched,
// write compact per-token records (conv input; normalised k, v, g, beta) and
// the NEXT call first replays `pending[slot]` records into the committed
// state (the reference's deferred-commit design for GDN MTP verify,
// reference: suffix_hybrid/kernels/gdn_defer_rocm.py).  Math per token and
// v-head (reference: src/qwen_gdn.rs:17-38):
//   q, k = l2norm(q), l2norm(k); q *= K^-1/2
//   g = -exp(A_log) * softplus(a + dt_bias); beta = sigmoid(b)
//   S = S * exp(g); v' = beta (v - S k); S = S + v' k^T; o = S q
//   out = rms_norm(o) * w * silu(z)
//
// gdn_conv:      one thread per (request, channel): KW-1 = 3 state taps kept
//                in registers; SiLU(causal depthwise conv).
// gdn_recurrent: one CTA per (request, v-head), thread v owns state row
//                S[v, 0:K] in registers; the shared q/k vectors and gates are
//                staged in shared memory per token.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gdn.h"
#include "pdl.cuh"

namespace shk {
namespace gdn {

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

__device__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < static_cast<int>((blockDim.x + 31) >> 5); ++i) t += red[i];
  return t;
}

// x: pre-conv activations [T, C] (row stride x_stride); y: [T, C] SiLU(conv).
// state [slots, C, KW-1] fp32; rec_x [slots, W, C] fp32 window inputs.
__global__ void conv_kernel(GdnConvParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int b = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= p.C) return;
  const int64_t slot = p.slots[b];
  const int64_t t0 = p.q_start[b], t1 = p.q_start[b + 1];
  float* st = p.state + (slot * p.C + c) * 3;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f;  // oldest .. newest
  if (p.mode == 1) {
    s0 = st[0];
    s1 = st[1];
    s2 = st[2];
    const int n = p.pending ? p.pending[slot] : 0;
    for (int i = 0; i < n; ++i) {
      const float xi = p.rec_x[(slot * p.W + i) * p.C + c];
      s0 = s1;
      s1 = s2;
      s2 = xi;
    }
    if (n > 0) {
      st[0] = s0;
      st[1] = s1;
      st[2] = s2;
    }
  }
  const float w0 = p.w[c * 4 + 0], w1 = p.w[c * 4 + 1], w2 = p.w[c * 4 + 2], w3 = p.w[c * 4 + 3];
  float a0 = s0, a1 = s1, a2 = s2;
  for (int64_t t = t0; t < t1; ++t) {
    const float xt = bf(p.x[t * p.x_stride + c]);
    const float acc = a0 * w0 + a1 * w1 + a2 * w2 + xt * w3;
    p.y[t * p.C + c] = __float2bfloat16(silu(acc));
    if (p.mode == 1) p.rec_x[(slot * p.W + (t - t0)) * p.C + c] = xt;
    a0 = a1;
    a1 = a2;
    a2 = xt;
  }
  if (p.mode == 0) {  // prefill commits its final taps
    st[0] = a0;
    st[1] = a1;
    st[2] = a2;
  }
}

template <int K>
__global__ void __launch_bounds__(K) recurrent_kernel(GdnParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  // Requires K == V == blockDim.x (checked on the host).
  __shared__ float sk[K], sq[K], red[32];
  __shared__ float sg, sb;
  const int b = blockIdx.x, hv = blockIdx.y, v = threadIdx.x;
  const int h = hv / (p.HV / p.H);
  const int64_t slot = p.slots[b];
  const int64_t t0 = p.q_start[b], t1 = p.q_start[b + 1];
  float* Srow = p.state + ((slot * p.HV + hv) * K + v) * K;
  float s[K];
  if (p.mode == 0) {
#pragma unroll
    for (int i = 0; i < K; ++i) s[i] = 0.f;
  } else {
#pragma unroll
    for (int i = 0; i < K; i += 4) {
      const float4 f = reinterpret_cast<const float4*>(Srow)[i / 4];
      s[i] = f.x;
      s[i + 1] = f.y;
      s[i + 2] = f.z;
      s[i + 3] = f.w;
    }
    // Deferred commit: replay the accepted tokens of the previous window.
    const int n = p.pending ? p.pending[slot] : 0;
    for (int r = 0; r < n; ++r) {
      const int64_t rec = (slot * p.W + r) * p.HV + hv;
      __syncthreads();
      sk[v] = p.rec_k[rec * K + v];
      if (v == 0) {
        sg = p.rec_g[rec];
        sb = p.rec_b[rec];
      }
      __syncthreads();
      const float eg = __expf(sg);
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < K; ++i) {
        s[i] *= eg;
        dot += s[i] * sk[i];
      }
      const float vp = sb * (p.rec_v[rec * K + v] - dot);
#pragma unroll
      for (int i = 0; i < K; ++i) s[i] += vp * sk[i];
    }
    if (n > 0) {
#pragma unroll
      for (int i = 0; i < K; i += 4)
        reinterpret_cast<float4*>(Srow)[i / 4] = make_float4(s[i], s[i + 1], s[i + 2], s[i + 3]);
    }
  }
  const float qscale = rsqrtf(static_cast<float>(K));
  for (int64_t t = t0; t < t1; ++t) {
    const __nv_bfloat16* row = p.qkv + t * p.qkv_stride;
    const float qv = bf(row[h * K + v]);
    const float kv = bf(row[p.H * K + h * K + v]);
    const float vv = bf(row[2 * p.H * K + hv * K + v]);
    const float qss = block_sum(qv * qv, red);
    const float kss = block_sum(kv * kv, red);
    __syncthreads();
    sq[v] = qv * rsqrtf(qss + 1e-6f) * qscale;
    sk[v] = kv * rsqrtf(kss + 1e-6f);
    if (v == 0) {
      const float bb = bf(p.ba[t * p.ba_stride + hv]);
      const float aa = bf(p.ba[t * p.ba_stride + p.HV + hv]);
      sg = -__expf(p.a_log[hv]) * softplus(aa + p.dt_bias[hv]);
      sb = 1.f / (1.f + __expf(-bb));
    }
    __syncthreads();
    const float eg = __expf(sg);
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < K; ++i) {
      s[i] *= eg;
      dot += s[i] * sk[i];
    }
    const float vp = sb * (vv - dot);
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < K; ++i) {
      s[i] += vp * sk[i];
      o += s[i] * sq[i];
    }
    if (p.mode == 1) {
      const int64_t rec = (slot * p.W + (t - t0)) * p.HV + hv;
      p.rec_k[rec * K + v] = sk[v];
      p.rec_v[rec * K + v] = vv;
      if (v == 0) {
        p.rec_g[rec] = sg;
        p.rec_b[rec] = sb;
      }
    }
    // Gated RMSNorm over the V outputs of this head.
    const float oss = block_sum(o * o, red);
    const float inv = rsqrtf(oss / K + p.eps);
    const float zz = bf(p.z[t * p.z_stride + hv * K + v]);
    p.out[t * p.out_stride + hv * K + v] = __float2bfloat16(o * inv * bf(p.norm_w[v]) * silu(zz));
  }
  if (p.mode == 0) {
#pragma unroll
    for (int i = 0; i < K; i += 4)
      reinterpret_cast<float4*>(Srow)[i / 4] = make_float4(s[i], s[i + 1], s[i + 2], s[i + 3]);
  }
}

}  // namespace gdn
}  // namespace shk

using namespace shk::gdn;

extern "C" int sh_gdn_conv(const GdnConvParams* p, int batch, cudaStream_t stream) {
  if (batch <= 0) return 0;
  if (p->KW != 4) return -1;
  dim3 grid((p->C + 127) / 128, batch);
  shk::launch(conv_kernel, dim3(grid), dim3(128), 0, stream, *p);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_gdn_recurrent(const GdnParams* p, int batch, cudaStream_t stream) {
  if (batch <= 0) return 0;
  if (p->K != p->V || p->HV % p->H != 0) return -1;
  dim3 grid(batch, p->HV);
  switch (p->K) {
    case 32:
      shk::launch(recurrent_kernel<32>, dim3(grid), dim3(32), 0, stream, *p);
      break;
    case 64:
      shk::launch(recurrent_kernel<64>, dim3(grid), dim3(64), 0, stream, *p);
      break;
    case 128:
      shk::launch(recurrent_kernel<128>, dim3(grid), dim3(128), 0, stream, *p);
      break;
    default:
      return -2;
  }
  return static_cast<int>(cudaGetLastError());
}
