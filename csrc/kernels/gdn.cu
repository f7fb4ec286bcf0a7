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
// gdn_recurrent: one CTA per (request, v-head), the state in registers
//                (K = 128: 256 threads, 4 rows x 16 columns each; K = 32 / 64:
//                4 threads per row); tokens staged in shared memory in chunks
//                with two barriers per chunk.
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

// Four threads per state row.  Thread t of the CTA owns row v = t / 4 and the
// K/4 columns {16 m + 4 j + c : j = t % 4, c < 4}: every state load is a
// 64-byte run per row, the q / k reads from shared memory are float4
// broadcasts, and the two dot products per token reduce with two shuffles.
// Tokens are processed in chunks of CH = K/16: in phase 1 warp pair c
// normalises token c (warp 2c: q and the output gate z, warp 2c+1: k, v and
// the gates) into shared memory; phase 2 runs the CH recurrent steps with no
// barrier; phase 3 (warp 2c) applies the gated RMSNorm of token c.  The next
// chunk's inputs are loaded into registers before phase 2 so their latency
// hides behind the recurrence.
// Copies n bf16 elements (n = K / 32 per lane) from global to shared memory:
// cp.async (no registers held while in flight) when the source is aligned to
// the copy size, plain loads otherwise.
template <int N>
__device__ __forceinline__ void stage_copy(__nv_bfloat16* dst, const __nv_bfloat16* src, bool async_ok) {
  constexpr int BYTES = N * 2;
  if constexpr (BYTES == 4 || BYTES == 8 || BYTES == 16) {
    if (async_ok) {
      const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
      asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(d), "l"(src), "n"(BYTES));
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < N; ++e) dst[e] = src[e];
}

__device__ __forceinline__ void stage_commit() { asm volatile("cp.async.commit_group;"); }
__device__ __forceinline__ void stage_wait() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Shared-memory float4 load the compiler may not merge with an earlier one:
// the update loop re-reads k instead of keeping K/4 values live across the dot.
__device__ __forceinline__ float4 lds4(const float* ptr) {
  float4 r;
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "r"(a));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int K, int TPR, int MINB>
__global__ void __launch_bounds__(TPR * K, MINB) recurrent_kernel(GdnParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  // TPR threads per state row, each owning NF4 float4 column groups; CH tokens per chunk.
  constexpr int NW = TPR * K / 32, CH = NW / 2 < 8 ? NW / 2 : 8, EPL = K / 32, NF4 = K / (4 * TPR);
  __shared__ __align__(16) float qn[CH][K], kn[CH][K], vs[CH][K], os[CH][K], zs[CH][K];
  __shared__ float gs[CH], bs[CH];
  // Raw inputs of the next chunk, double-buffered: [buffer][token][role][q|k , z|v][K].
  __shared__ __align__(16) __nv_bfloat16 stg[2][CH][2][2][K];
  __shared__ __align__(8) uint32_t gst[2][CH][2];  // aligned 4-byte words holding the b and a gate inputs
  const int b = blockIdx.x, hv = blockIdx.y;
  const int tid = threadIdx.x, row = tid / TPR, j = tid % TPR;
  const int warp = tid >> 5, lane = tid & 31, tc = warp >> 1, role = warp & 1;
  const int h = hv / (p.HV / p.H);
  const int slot = static_cast<int>(p.slots[b]);
  const int t0 = static_cast<int>(p.q_start[b]);
  const int ntok = static_cast<int>(p.q_start[b + 1]) - t0;
  const float qscale = rsqrtf(static_cast<float>(K));
  float4* Srow = reinterpret_cast<float4*>(p.state + ((static_cast<int64_t>(slot) * p.HV + hv) * K + row) * K) + j;
  float4 s[NF4];
  if (p.mode == 0) {
#pragma unroll
    for (int m = 0; m < NF4; ++m) s[m] = make_float4(0.f, 0.f, 0.f, 0.f);
  } else {
#pragma unroll
    for (int m = 0; m < NF4; ++m) s[m] = Srow[TPR * m];
  }

  // One recurrent step on token slot c of the staged chunk; returns this row's S q.
  auto step = [&](int c, bool want_o) -> float {
    const float eg = __expf(gs[c]);
    const float* kk = kn[c] + 4 * j;
    constexpr int CS = 4 * TPR;  // column stride between a thread's float4 groups
    float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
    for (int m = 0; m < NF4; ++m) {
      const float4 k4 = lds4(kk + CS * m);
      s[m].x *= eg; s[m].y *= eg; s[m].z *= eg; s[m].w *= eg;
      d0 += s[m].x * k4.x; d1 += s[m].y * k4.y; d2 += s[m].z * k4.z; d3 += s[m].w * k4.w;
    }
    float dot = (d0 + d1) + (d2 + d3);
#pragma unroll
    for (int x = 1; x < TPR; x <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, x);
    const float vp = bs[c] * (vs[c][row] - dot);
    const float* qq = qn[c] + 4 * j;
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
    for (int m = 0; m < NF4; ++m) {
      const float4 k4 = lds4(kk + CS * m);
      s[m].x += vp * k4.x; s[m].y += vp * k4.y; s[m].z += vp * k4.z; s[m].w += vp * k4.w;
      if (want_o) {
        const float4 q4 = lds4(qq + CS * m);
        o0 += s[m].x * q4.x; o1 += s[m].y * q4.y; o2 += s[m].z * q4.z; o3 += s[m].w * q4.w;
      }
    }
    float o = (o0 + o1) + (o2 + o3);
    if (want_o) {
#pragma unroll
      for (int x = 1; x < TPR; x <<= 1) o += __shfl_xor_sync(0xffffffffu, o, x);
    }
    return o;
  };

  auto load_tok = [&](int c0, int buf) {
    const int c = c0 + tc;
    if (tc >= CH || c >= ntok) return;
    const int64_t t = t0 + c;
    const __nv_bfloat16* qkv = p.qkv + t * p.qkv_stride;
    __nv_bfloat16* d0 = &stg[buf][tc][role][0][lane * EPL];
    __nv_bfloat16* d1 = &stg[buf][tc][role][1][lane * EPL];
    if (role == 0) {
      stage_copy<EPL>(d0, qkv + h * K + lane * EPL, p.async_ok);
      stage_copy<EPL>(d1, p.z + t * p.z_stride + hv * K + lane * EPL, p.async_ok);
    } else {
      stage_copy<EPL>(d0, qkv + p.H * K + h * K + lane * EPL, p.async_ok);
      stage_copy<EPL>(d1, qkv + 2 * p.H * K + hv * K + lane * EPL, p.async_ok);
      if (lane < 2) {  // lane 0: b, lane 1: a (the aligned word that holds it)
        const int64_t i = t * p.ba_stride + hv + lane * p.HV;
        const __nv_bfloat16* src = p.ba + (i & ~int64_t(1));
        if (p.async_ok) {
          const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(&gst[buf][tc][lane]));
          asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src));
        } else {
          gst[buf][tc][lane] = *reinterpret_cast<const uint32_t*>(src);
        }
      }
    }
    stage_commit();
  };
  load_tok(0, 0);
  // Deferred commit: replay the accepted records of the previous window into the committed state.
  const int npend = (p.mode == 1 && p.pending) ? p.pending[slot] : 0;
  for (int r0 = 0; r0 < npend; r0 += CH) {
    const int n = min(CH, npend - r0);
    if (role == 1 && tc < n) {  // n <= CH
      const int64_t rec = (slot * p.W + r0 + tc) * p.HV + hv;
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        kn[tc][lane * EPL + e] = p.rec_k[rec * K + lane * EPL + e];
        vs[tc][lane * EPL + e] = p.rec_v[rec * K + lane * EPL + e];
      }
      if (lane == 0) {
        gs[tc] = p.rec_g[rec];
        bs[tc] = p.rec_b[rec];
      }
    }
    __syncthreads();
    for (int c = 0; c < n; ++c) step(c, false);
    __syncthreads();
  }
  if (npend > 0) {
#pragma unroll
    for (int m = 0; m < NF4; ++m) Srow[TPR * m] = s[m];
  }

  for (int c0 = 0, buf = 0; c0 < ntok; c0 += CH, buf ^= 1) {
    const int n = min(CH, ntok - c0);
    if (tc < n) {  // phase 1: normalise token c0 + tc into slot tc
      stage_wait();
      __syncwarp();  // lane 0 reads the gate word lane 1 staged
      float ra[EPL], rb[EPL], ss = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        ra[e] = bf(stg[buf][tc][role][0][lane * EPL + e]);
        rb[e] = bf(stg[buf][tc][role][1][lane * EPL + e]);
        ss += ra[e] * ra[e];
      }
      const float inv = rsqrtf(warp_sum(ss) + 1e-6f);
      if (role == 0) {
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          qn[tc][lane * EPL + e] = ra[e] * inv * qscale;
          zs[tc][lane * EPL + e] = rb[e];
        }
      } else {
        const int64_t rec = (slot * p.W + c0 + tc) * p.HV + hv;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float kv = ra[e] * inv;
          kn[tc][lane * EPL + e] = kv;
          vs[tc][lane * EPL + e] = rb[e];
          if (p.mode == 1) {
            p.rec_k[rec * K + lane * EPL + e] = kv;
            p.rec_v[rec * K + lane * EPL + e] = rb[e];
          }
        }
        if (lane == 0) {
          const int64_t i = static_cast<int64_t>(t0 + c0 + tc) * p.ba_stride + hv;
          const uint32_t wb = gst[buf][tc][0], wa = gst[buf][tc][1];
          const float gb = __uint_as_float(((i & 1) ? (wb >> 16) : (wb & 0xffffu)) << 16);
          const float ga = __uint_as_float((((i + p.HV) & 1) ? (wa >> 16) : (wa & 0xffffu)) << 16);
          const float g = -__expf(p.a_log[hv]) * softplus(ga + p.dt_bias[hv]);
          const float be = 1.f / (1.f + __expf(-gb));
          gs[tc] = g;
          bs[tc] = be;
          if (p.mode == 1) {
            p.rec_g[rec] = g;
            p.rec_b[rec] = be;
          }
        }
      }
    }
    __syncthreads();
    load_tok(c0 + CH, buf ^ 1);  // prefetch the next chunk behind the recurrence
    for (int c = 0; c < n; ++c) {  // phase 2
      const float o = step(c, true);
      if (j == 0) os[c][row] = o;
    }
    __syncthreads();
    if (role == 0 && tc < n) {  // phase 3: gated RMSNorm of token c0 + tc
      const int64_t t = t0 + c0 + tc;
      float o[EPL], ss = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        o[e] = os[tc][lane * EPL + e];
        ss += o[e] * o[e];
      }
      const float inv = rsqrtf(warp_sum(ss) / K + p.eps);
      __nv_bfloat16* dst = p.out + t * p.out_stride + hv * K + lane * EPL;
#pragma unroll
      for (int e = 0; e < EPL; ++e)
        dst[e] = __float2bfloat16(o[e] * inv * bf(p.norm_w[lane * EPL + e]) * silu(zs[tc][lane * EPL + e]));
    }
  }
  if (p.mode == 0) {
#pragma unroll
    for (int m = 0; m < NF4; ++m) Srow[TPR * m] = s[m];
  }
}

// K = 128 path: one 256-thread CTA per (request, v-head).  Thread (warp w,
// lane l) owns rows 16w + 4(l/8) + {0..3} and the 16 columns
// {32 m + 4 (l % 8) + c}: one k / q value from shared memory feeds four rows,
// and a row reduces over 8 lanes.  The decay is kept as a running scalar
// (S = c * S~, renormalised per chunk or when c would underflow) and
// o = S_new q is formed from the old state as eg c (S~ q) + vp (k . q), so a
// token costs 3 FMAs per state element: S~ k, S~ q and the rank-1 update.
template <int BYTES>
__device__ __forceinline__ void cp_async(void* dst, const void* src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(d), "l"(src), "n"(BYTES));
}

__global__ void __launch_bounds__(256, 2) recurrent_head_kernel(GdnParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  constexpr int K = 128, CH = 8, NF4 = 4, R = 4;
  __shared__ __align__(16) float qn[CH][K], kn[CH][K], vs[CH][K], zs[CH][K], os[CH][K];
  __shared__ float gs[CH], bs[CH], kqs[CH];
  // Raw inputs of the next chunk, double-buffered: [buffer][token][q | k | v | z][K].
  __shared__ __align__(16) __nv_bfloat16 stg[2][CH][4][K];
  __shared__ __align__(8) uint32_t gst[2][CH][2];
  const int b = blockIdx.x, hv = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, cl = lane & 7;
  const int row0 = warp * 16 + (lane >> 3) * R;
  const int h = hv / (p.HV / p.H);
  const int slot = static_cast<int>(p.slots[b]);
  const int t0 = static_cast<int>(p.q_start[b]);
  const int ntok = static_cast<int>(p.q_start[b + 1]) - t0;
  const float qscale = rsqrtf(static_cast<float>(K));
  const bool ok = p.async_ok != 0;
  float4* Sg = reinterpret_cast<float4*>(p.state + ((static_cast<int64_t>(slot) * p.HV + hv) * K + row0) * K) + cl;
  float4 s[R][NF4];
  float cs = 1.f;  // S = cs * s
  const int npend = (p.mode == 1 && p.pending) ? p.pending[slot] : 0;

  auto load_rec = [&](int r0) {  // records r0 + warp -> kn / vs / gs / bs
    const int r = r0 + warp;
    if (warp >= CH || r >= npend) return;
    const int64_t rec = (static_cast<int64_t>(slot) * p.W + r) * p.HV + hv;
    cp_async<16>(&kn[warp][lane * 4], p.rec_k + rec * K + lane * 4);
    cp_async<16>(&vs[warp][lane * 4], p.rec_v + rec * K + lane * 4);
    if (lane == 0) cp_async<4>(&gs[warp], p.rec_g + rec);
    if (lane == 1) cp_async<4>(&bs[warp], p.rec_b + rec);
  };
  auto load_tok = [&](int c0, int buf) {
    const int c = c0 + warp;
    if (warp >= CH || c >= ntok) return;
    const int64_t t = t0 + c;
    const __nv_bfloat16* qkv = p.qkv + t * p.qkv_stride;
    const __nv_bfloat16* src[4] = {qkv + h * K + lane * 4, qkv + p.H * K + h * K + lane * 4,
                                   qkv + 2 * p.H * K + hv * K + lane * 4, p.z + t * p.z_stride + hv * K + lane * 4};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (ok) {
        cp_async<8>(&stg[buf][warp][i][lane * 4], src[i]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) stg[buf][warp][i][lane * 4 + e] = src[i][e];
      }
    }
    if (lane < 2) {  // lane 0: b, lane 1: a (the aligned 4-byte word that holds it)
      const int64_t i = t * p.ba_stride + hv + lane * p.HV;
      const __nv_bfloat16* w = p.ba + (i & ~int64_t(1));
      if (ok)
        cp_async<4>(&gst[buf][warp][lane], w);
      else
        gst[buf][warp][lane] = *reinterpret_cast<const uint32_t*>(w);
    }
  };

  if (p.mode == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < NF4; ++m) s[r][m] = make_float4(0.f, 0.f, 0.f, 0.f);
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < NF4; ++m) s[r][m] = Sg[r * (K / 4) + 8 * m];
  }
  if (ok) load_rec(0);
  load_tok(0, 0);
  asm volatile("cp.async.commit_group;");

  auto rescale = [&](float f) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < NF4; ++m) {
        s[r][m].x *= f; s[r][m].y *= f; s[r][m].z *= f; s[r][m].w *= f;
      }
  };
  // One token on staged slot c; with want_o the rows' S_new q go to os[c].
  auto step = [&](int c, bool want_o) {
    float ceg = cs * __expf(gs[c]);
    if (ceg < 1e-20f) {  // uniform over the CTA: fold the scale in before it underflows
      rescale(ceg);
      ceg = 1.f;
    }
    const float* kk = kn[c] + 4 * cl;
    const float* qq = qn[c] + 4 * cl;
    float d[R], e[R];
#pragma unroll
    for (int r = 0; r < R; ++r) d[r] = e[r] = 0.f;
#pragma unroll
    for (int m = 0; m < NF4; ++m) {
      const float4 k4 = lds4(kk + 32 * m);
#pragma unroll
      for (int r = 0; r < R; ++r) d[r] += s[r][m].x * k4.x + s[r][m].y * k4.y + s[r][m].z * k4.z + s[r][m].w * k4.w;
      if (want_o) {
        const float4 q4 = lds4(qq + 32 * m);
#pragma unroll
        for (int r = 0; r < R; ++r)
          e[r] += s[r][m].x * q4.x + s[r][m].y * q4.y + s[r][m].z * q4.z + s[r][m].w * q4.w;
      }
    }
#pragma unroll
    for (int x = 1; x < 8; x <<= 1)
#pragma unroll
      for (int r = 0; r < R; ++r) d[r] += __shfl_xor_sync(0xffffffffu, d[r], x);
    const float4 v4 = *reinterpret_cast<const float4*>(&vs[c][row0]);
    const float beta = bs[c];
    float vp[R];
    vp[0] = beta * (v4.x - ceg * d[0]);
    vp[1] = beta * (v4.y - ceg * d[1]);
    vp[2] = beta * (v4.z - ceg * d[2]);
    vp[3] = beta * (v4.w - ceg * d[3]);
    if (want_o) {  // transpose-reduce over the 8 lanes of a row group: lane cl = 2 r ends with row r
      const bool b2 = (cl & 4) != 0, b1 = (cl & 2) != 0;
      float x0 = (b2 ? e[2] : e[0]) + __shfl_xor_sync(0xffffffffu, b2 ? e[0] : e[2], 4);
      float x1 = (b2 ? e[3] : e[1]) + __shfl_xor_sync(0xffffffffu, b2 ? e[1] : e[3], 4);
      float y = (b1 ? x1 : x0) + __shfl_xor_sync(0xffffffffu, b1 ? x0 : x1, 2);
      y += __shfl_xor_sync(0xffffffffu, y, 1);
      if ((cl & 1) == 0) {
        const int r = (b2 ? 2 : 0) + (b1 ? 1 : 0);
        os[c][row0 + r] = ceg * y + vp[r] * kqs[c];
      }
    }
    const float inv = 1.f / ceg;
#pragma unroll
    for (int m = 0; m < NF4; ++m) {
      const float4 k4 = lds4(kk + 32 * m);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float u = vp[r] * inv;
        s[r][m].x += u * k4.x; s[r][m].y += u * k4.y; s[r][m].z += u * k4.z; s[r][m].w += u * k4.w;
      }
    }
    cs = ceg;
  };
  auto store_state = [&]() {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < NF4; ++m) Sg[r * (K / 4) + 8 * m] = s[r][m];
  };

  // Deferred commit: replay the accepted records of the previous window into the committed state.
  for (int r0 = 0; r0 < npend; r0 += CH) {
    if (r0 > 0 || !ok) {
      __syncthreads();  // the previous chunk's steps are done with kn / vs
      if (ok) {
        load_rec(r0);
        asm volatile("cp.async.commit_group;");
      } else if (warp < CH && r0 + warp < npend) {
        const int64_t rec = (static_cast<int64_t>(slot) * p.W + r0 + warp) * p.HV + hv;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          kn[warp][lane * 4 + e] = p.rec_k[rec * K + lane * 4 + e];
          vs[warp][lane * 4 + e] = p.rec_v[rec * K + lane * 4 + e];
        }
        if (lane == 0) {
          gs[warp] = p.rec_g[rec];
          bs[warp] = p.rec_b[rec];
        }
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    const int n = min(CH, npend - r0);
    for (int c = 0; c < n; ++c) step(c, false);
  }
  if (npend > 0) {
    rescale(cs);
    cs = 1.f;
    store_state();
  }
  __syncthreads();  // replay done with kn / vs / gs / bs

  for (int c0 = 0, buf = 0; c0 < ntok; c0 += CH, buf ^= 1) {
    const int n = min(CH, ntok - c0);
    if (warp < n) {  // phase 1: token c0 + warp -> slot warp
      asm volatile("cp.async.wait_group 0;" ::: "memory");
      __syncwarp();  // lane 0 reads the gate word lane 1 staged
      float q[4], k[4], v[4], z[4], qs = 0.f, ks = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        q[e] = bf(stg[buf][warp][0][lane * 4 + e]);
        k[e] = bf(stg[buf][warp][1][lane * 4 + e]);
        v[e] = bf(stg[buf][warp][2][lane * 4 + e]);
        z[e] = bf(stg[buf][warp][3][lane * 4 + e]);
        qs += q[e] * q[e];
        ks += k[e] * k[e];
      }
      const float iq = rsqrtf(warp_sum(qs) + 1e-6f) * qscale, ik = rsqrtf(warp_sum(ks) + 1e-6f);
      float kq = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        q[e] *= iq;
        k[e] *= ik;
        kq += q[e] * k[e];
      }
      const float4 q4 = make_float4(q[0], q[1], q[2], q[3]), k4 = make_float4(k[0], k[1], k[2], k[3]);
      const float4 v4 = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(&qn[warp][lane * 4]) = q4;
      *reinterpret_cast<float4*>(&kn[warp][lane * 4]) = k4;
      *reinterpret_cast<float4*>(&vs[warp][lane * 4]) = v4;
      *reinterpret_cast<float4*>(&zs[warp][lane * 4]) = make_float4(z[0], z[1], z[2], z[3]);
      const int64_t rec = (static_cast<int64_t>(slot) * p.W + c0 + warp) * p.HV + hv;
      if (p.mode == 1) {
        *reinterpret_cast<float4*>(p.rec_k + rec * K + lane * 4) = k4;
        *reinterpret_cast<float4*>(p.rec_v + rec * K + lane * 4) = v4;
      }
      kq = warp_sum(kq);
      if (lane == 0) {
        const int64_t i = static_cast<int64_t>(t0 + c0 + warp) * p.ba_stride + hv;
        const uint32_t wb = gst[buf][warp][0], wa = gst[buf][warp][1];
        const float gb = __uint_as_float(((i & 1) ? (wb >> 16) : (wb & 0xffffu)) << 16);
        const float ga = __uint_as_float((((i + p.HV) & 1) ? (wa >> 16) : (wa & 0xffffu)) << 16);
        const float g = -__expf(p.a_log[hv]) * softplus(ga + p.dt_bias[hv]);
        const float be = 1.f / (1.f + __expf(-gb));
        gs[warp] = g;
        bs[warp] = be;
        kqs[warp] = kq;
        if (p.mode == 1) {
          p.rec_g[rec] = g;
          p.rec_b[rec] = be;
        }
      }
    }
    __syncthreads();
    load_tok(c0 + CH, buf ^ 1);  // prefetch the next chunk behind the recurrence
    asm volatile("cp.async.commit_group;");
    for (int c = 0; c < n; ++c) step(c, true);
    rescale(cs);
    cs = 1.f;
    __syncthreads();
    if (warp < n) {  // phase 3: gated RMSNorm of token c0 + warp over the head's 128 rows
      const float4 o4 = *reinterpret_cast<const float4*>(&os[warp][lane * 4]);
      const float o[4] = {o4.x, o4.y, o4.z, o4.w};
      const float inv = rsqrtf(warp_sum(o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3]) / K + p.eps);
      const int64_t t = t0 + c0 + warp;
      __nv_bfloat16* dst = p.out + t * p.out_stride + hv * K + lane * 4;
      float r[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) r[e] = o[e] * inv * bf(p.norm_w[lane * 4 + e]) * silu(zs[warp][lane * 4 + e]);
      const __nv_bfloat162 lo = __floats2bfloat162_rn(r[0], r[1]), hi = __floats2bfloat162_rn(r[2], r[3]);
      uint2 u;
      u.x = *reinterpret_cast<const uint32_t*>(&lo);
      u.y = *reinterpret_cast<const uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(dst) = u;
    }
  }
  if (p.mode == 0) store_state();
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
  GdnParams q = *p;
  const int cpy = (p->K / 32) * 2;  // bytes per lane per staged row
  auto al = [&](const void* ptr, int64_t stride) {
    return reinterpret_cast<uintptr_t>(ptr) % cpy == 0 && (stride * 2) % cpy == 0;
  };
  q.async_ok = al(p->qkv, p->qkv_stride) && al(p->z, p->z_stride) && ((p->H * p->K * 2) % cpy == 0) &&
                reinterpret_cast<uintptr_t>(p->ba) % 4 == 0 ? 1 : 0;
  dim3 grid(batch, p->HV);
  switch (p->K) {
    case 32:
      shk::launch(recurrent_kernel<32, 4, 2>, dim3(grid), dim3(128), 0, stream, q);
      break;
    case 64:
      shk::launch(recurrent_kernel<64, 4, 2>, dim3(grid), dim3(256), 0, stream, q);
      break;
    case 128:
      shk::launch(recurrent_head_kernel, dim3(grid), dim3(256), 0, stream, q);
      break;
    default:
      return -2;
  }
  return static_cast<int>(cudaGetLastError());
}
