// Chunked Gated DeltaNet prefill on the tcgen05 tensor cores (K = V = 128,
// chunk C = 64), from zero state: one CTA per (request, v-head) walks its
// request's chunks in order with the fp32 state in TMEM.
//
// Per chunk, with b_t = exp(gamma_t) the in-chunk cumulative decay (all
// decay ratios below are exp(gamma_t - gamma_j) <= 1), the recurrence of
// csrc/kernels/gdn.cu is evaluated in the WY form
//   L[t,j]  = beta_t e^{g_t-g_j} k_t.k_j  (j < t),   T = (I + L)^-1
//   W = T diag(beta b) K,  U = T diag(beta) V,  D = U - W S0^T
//   O = diag(b) Q S0^T + Mq D,   Mq[t,j] = e^{g_t-g_j} q_t.k_j  (j <= t)
//   S_C = b_C S0 + D^T diag(b_C / b) K
// (reference math: src/qwen_gdn.rs:17-38; chunk size 64 as in the Qwen3-Next
// serving configuration).  The tensor-core products, all M = 128, bf16
// operands in 128-byte-swizzled K-major shared tiles, fp32 in TMEM:
//   MMA1  [K; Q] . K^T                  -> [G; QK]           (64 columns)
//   MMA5  [T diag(beta b); T diag(beta)] . [K^T; V^T]^T -> W, U (256 columns)
//   MMA4  [Q; W] . S0^T                 -> [Q S0^T; W S0^T]  (128 columns)
//   MMA6  [Mq; -] . D                   -> Mq D              (128 columns)
//   MMA7  X += (D^T diag(b_C/b)) . K    -> state             (128 columns)
// The unit lower-triangular inverse T is done in fp32 on the CUDA cores in
// 16 x 16 blocks.  The state X in TMEM is pre-scaled by b_C of the chunk
// before MMA7 accumulates into it (in the previous chunk's state pass, with
// that chunk's gates computed ahead), and its bf16 copy (the S0 operand of the
// next chunk) is written after.  The next chunk's raw rows are prefetched with
// cp.async while the output phase runs.  Rows past the request's last token are
// zero: they add nothing to the state and their outputs are not stored.
//
// Roles are phase-sequential (all 256 threads, barriers between phases);
// every warp-collective tcgen05 instruction (.sync.aligned) runs on whole
// warps, also in the last, partial chunk;
// thread 0 issues each MMA group and commits it to one mbarrier.  Every
// mbarrier wait is bounded: on timeout the kernel records an error, waits
// (bounded) for the MMA in flight, frees its TMEM and returns.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gdn.h"
#include "pdl.cuh"
#include "tcgen05_common.cuh"

namespace shk {
namespace gdnc {

using namespace shk::tc;

constexpr int C = 64, K = 128, NT = 256;

// Shared memory (bytes).  Operand tiles are 1024-byte aligned 128-byte-swizzled
// K-major atoms of 64 bf16 columns.
constexpr int X_ATOM = 192 * 128;  // rows 0-63 K, 64-127 Q, 128-191 W
constexpr int OFF_X = 0;           // two atoms (columns 0-63, 64-127)
constexpr int S_ATOM = 128 * 128;  // S0 bf16 [v][k]
constexpr int OFF_S = OFF_X + 2 * X_ATOM;
constexpr int OFF_KVT = OFF_S + 2 * S_ATOM;  // rows 0-127 K^T [k][j], 128-255 V^T [v][j]
constexpr int OFF_B12 = OFF_KVT + 256 * 128;  // rows 0-63 T diag(beta b), 64-127 T diag(beta)
constexpr int OFF_MQ = OFF_B12 + 128 * 128;   // rows 0-63 Mq (rows 64-127 unused)
constexpr int OFF_DT = OFF_MQ + 128 * 128;    // D^T [v][j]
constexpr int OFF_A7 = OFF_DT + 128 * 128;    // D^T diag(b_C / b) [v][j]
// fp32 work arrays of the inverse share the D^T / A7 tiles (dead by then).
constexpr int LDF = 65;
constexpr int OFF_LF = OFF_DT;
constexpr int OFF_TF = OFF_LF + 64 * LDF * 4;
constexpr int OFF_YF = OFF_TF + 64 * LDF * 4;
constexpr int YF_BYTES = 3 * 16 * 17 * 4;
constexpr int OFF_Z = ((OFF_YF + YF_BYTES + 1023) / 1024) * 1024;  // z rows of the chunk, bf16 [64][128]
constexpr int OFF_GAM = OFF_Z + 64 * 256;   // gates of two chunks: [2][64] each
constexpr int OFF_BV = OFF_GAM + 2 * 64 * 4;
constexpr int OFF_BETA = OFF_BV + 2 * 64 * 4;
constexpr int OFF_NW = OFF_BETA + 2 * 64 * 4;  // norm weight, fp32 [128]
// Raw k | q | v rows of the next chunk (bf16 [3][64][128], 16-byte chunks swizzled by row), prefetched
// during the output phase into the B12 / Mq / D^T tiles, which are dead from MMA6/7 until the next MMA5.
constexpr int OFF_STG = OFF_B12;
static_assert(OFF_STG + 3 * 64 * 256 <= OFF_A7, "staging fits the dead tiles");
constexpr int OFF_PART = OFF_NW + 128 * 4;  // per-row partial sums of o^2, [2][64]
constexpr int OFF_BAR = OFF_PART + 2 * 64 * 4;
constexpr int SMEM_BYTES = OFF_BAR + 64;
constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack to align the base to 1024
static_assert(OFF_A7 + 128 * 128 <= OFF_Z, "inverse work arrays alias the D^T tiles");
static_assert(OFF_YF + YF_BYTES <= OFF_Z, "layout");
static_assert(SMEM_ALLOC <= 227 * 1024, "shared memory");

// TMEM columns: state X [0,128), MMA4 [128,256), MMA1 / MMA5 / MMA6 [256,512).
constexpr uint32_t TM_X = 0, TM_4 = 128, TM_5 = 256, TCOLS = 512;

__device__ __forceinline__ uint32_t swz(int row, int col) {  // byte offset of (row, col) in an atom
  return static_cast<uint32_t>(row * 128 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2);
}
__device__ __forceinline__ void fence_proxy() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15])
      : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ void st_chunk(uint8_t* base, uint32_t off, const float* v) {  // 8 bf16
  uint4 u;
  u.x = pack_bf16(v[0], v[1]);
  u.y = pack_bf16(v[2], v[3]);
  u.z = pack_bf16(v[4], v[5]);
  u.w = pack_bf16(v[6], v[7]);
  *reinterpret_cast<uint4*>(base + off) = u;
}
__device__ __forceinline__ void st_bf16(uint8_t* base, uint32_t off, float v) {
  *reinterpret_cast<__nv_bfloat16*>(base + off) = __float2bfloat16(v);
}
__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

// Loads one 128-wide bf16 row (16-byte aligned) into registers as 64 packed pairs.
__device__ __forceinline__ void load_row(const __nv_bfloat16* src, uint32_t (&r)[64]) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint4 u = s4[i];
    r[4 * i] = u.x;
    r[4 * i + 1] = u.y;
    r[4 * i + 2] = u.z;
    r[4 * i + 3] = u.w;
  }
}
__device__ __forceinline__ float lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

__global__ void __launch_bounds__(NT, 1) gdn_chunk_kernel(GdnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* Lf = reinterpret_cast<float*>(sm + OFF_LF);
  float* Tf = reinterpret_cast<float*>(sm + OFF_TF);
  float* Yf = reinterpret_cast<float*>(sm + OFF_YF);
  float* gam_all = reinterpret_cast<float*>(sm + OFF_GAM);
  float* bv_all = reinterpret_cast<float*>(sm + OFF_BV);
  float* betav_all = reinterpret_cast<float*>(sm + OFF_BETA);
  float* nw = reinterpret_cast<float*>(sm + OFF_NW);
  float* part = reinterpret_cast<float*>(sm + OFF_PART);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + OFF_BAR + 16);
  const uint32_t sbase = smem_addr(sm);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, quarter = warp & 3;
  const int b = blockIdx.x, hv = blockIdx.y;
  const int h = hv / (p.HV / p.H);

  shk::pdl_trigger();
  shk::pdl_wait();
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (tid < K) nw[tid] = __bfloat162float(p.norm_w[tid]);
  // S0 = 0 for the first chunk.
  for (int i = tid; i < 2 * S_ATOM / 16; i += NT) reinterpret_cast<uint4*>(sm + OFF_S)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy();
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_off = static_cast<uint32_t>(32 * quarter) << 16;

  const int64_t slot = p.slots[b];
  const int64_t t0 = p.q_start[b];
  const int ntok = static_cast<int>(p.q_start[b + 1] - t0);
  const int nchunks = (ntok + C - 1) / C;
  const float qscale = rsqrtf(static_cast<float>(K));
  const float alog = __expf(p.a_log[hv]), dtb = p.dt_bias[hv];
  uint32_t phase = 0;
  bool failed = false;

  // Commit the MMAs issued so far and wait for them (all threads, uniform outcome).
  auto sync_mma = [&]() -> bool {
    if (tid == 0) mma_commit(bar);
    const bool ok = mbar_wait(bar, phase, abort_flag);
    if (!ok) *abort_flag = 1;
    phase ^= 1;
    __syncthreads();
    fence_after();
    return *abort_flag == 0;
  };

  // Gates of chunk ci (one warp, two tokens per lane) and their in-chunk cumulative sum -> buffer ci & 1.
  auto gates = [&](int ci) {
    const int c0 = ci * C, n = min(C, ntok - c0), bb = (ci & 1) * 64;
    float g2[2], be2[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int t = 2 * lane + e;
      g2[e] = 0.f;
      be2[e] = 0.f;
      if (t < n) {
        const __nv_bfloat16* ba = p.ba + (t0 + c0 + t) * p.ba_stride;
        const float bq = __bfloat162float(ba[hv]), aa = __bfloat162float(ba[p.HV + hv]);
        g2[e] = -alog * softplus(aa + dtb);
        be2[e] = 1.f / (1.f + __expf(-bq));
      }
    }
    float s = g2[0] + g2[1];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    const float g1 = s, g0 = s - g2[1];
    gam_all[bb + 2 * lane] = g0;
    gam_all[bb + 2 * lane + 1] = g1;
    bv_all[bb + 2 * lane] = __expf(g0);
    bv_all[bb + 2 * lane + 1] = __expf(g1);
    betav_all[bb + 2 * lane] = be2[0];
    betav_all[bb + 2 * lane + 1] = be2[1];
  };
  // cp.async of chunk ci's raw k / q / v rows into the staging tiles (threads of warps 2, 3, 6, 7: 128
  // threads, 24 copies each); rows past the request are not loaded (phase 0 zeroes them).
  auto prefetch_rows = [&](int ci, int idx) {
    const int c0 = ci * C, n = min(C, ntok - c0);
    for (int i = idx; i < 3 * 64 * 16; i += 128) {
      const int kind = i / (64 * 16), t = (i / 16) % 64, ch = i % 16;
      if (t >= n) continue;
      const __nv_bfloat16* row = p.qkv + (t0 + c0 + t) * p.qkv_stride +
                                 (kind == 0 ? p.H * K + h * K : kind == 1 ? h * K : 2 * p.H * K + hv * K);
      const uint32_t d = sbase + OFF_STG + (kind * 64 + t) * 256 + ((ch ^ (t & 7)) << 4);
      asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(d), "l"(row + ch * 8));
    }
    asm volatile("cp.async.commit_group;");
  };
  const bool stager = warp == 2 || warp == 3 || warp == 6 || warp == 7;
  const int stage_idx = (warp & 1) * 32 + (warp >> 2) * 64 + lane;  // 0..127 over the four staging warps
  if (nchunks > 0) {
    if (warp == 4) gates(0);
    if (stager) {
      prefetch_rows(0, stage_idx);
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
  }
  __syncthreads();

  for (int ci = 0; ci < nchunks && !failed; ++ci) {
    const int c0 = ci * C;
    const int n = min(C, ntok - c0);
    const float* gam = gam_all + (ci & 1) * 64;
    const float* bv = bv_all + (ci & 1) * 64;
    const float* betav = betav_all + (ci & 1) * 64;
    // ---------------------------------------------------------------- phase 0: stage the chunk
    if (warp < 6) {
      const int t = tid & 63, kind = tid >> 6;  // 0: k, 1: q, 2: v
      const bool valid = t < n;
      uint32_t r[64];
      if (valid) {  // the row prefetched into the staging tiles
        const uint8_t* srow = sm + OFF_STG + (kind * 64 + t) * 256;
#pragma unroll
        for (int ch = 0; ch < 16; ++ch) {
          const uint4 u = *reinterpret_cast<const uint4*>(srow + ((ch ^ (t & 7)) << 4));
          r[4 * ch] = u.x;
          r[4 * ch + 1] = u.y;
          r[4 * ch + 2] = u.z;
          r[4 * ch + 3] = u.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) r[i] = 0u;
      }
      float scale = 1.f;
      if (kind < 2) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 64; ++i) ss += lo(r[i]) * lo(r[i]) + hi(r[i]) * hi(r[i]);
        scale = rsqrtf(ss + 1e-6f) * (kind == 1 ? qscale : 1.f);
      }
      if (kind < 2) {  // row t of K (tile rows 0-63) or Q (rows 64-127)
        const int trow = kind == 0 ? t : 64 + t;
#pragma unroll
        for (int ch = 0; ch < 16; ++ch) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            v[2 * e] = lo(r[4 * ch + e]) * scale;
            v[2 * e + 1] = hi(r[4 * ch + e]) * scale;
          }
          st_chunk(sm + OFF_X + (ch >> 3) * X_ATOM, swz(trow, (ch & 7) * 8), v);
        }
      }
      if (kind != 1) {  // column t of K^T (rows 0-127) or V^T (rows 128-255)
        const int rbase = kind == 0 ? 0 : 128;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          st_bf16(sm + OFF_KVT, swz(rbase + 2 * i, t), lo(r[i]) * scale);
          st_bf16(sm + OFF_KVT, swz(rbase + 2 * i + 1, t), hi(r[i]) * scale);
        }
      }
    } else if (warp == 7) {  // z rows of the chunk -> shared memory (read by phase 5)
      for (int i = lane; i < n * 16; i += 32) {
        const int t = i >> 4, ch = i & 15;
        const __nv_bfloat16* src = p.z + (t0 + c0 + t) * p.z_stride + hv * K + ch * 8;
        const uint32_t d = sbase + OFF_Z + t * 256 + ((ch ^ (t & 7)) << 4);  // swizzled: conflict-free row reads
        asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src));
      }
      asm volatile("cp.async.commit_group;");  // waited for in phase 5
    }
    fence_proxy();
    fence_before();
    __syncthreads();
    // MMA1: [K; Q] (rows 0-127) x K^T (rows 0-63) -> TMEM [G; QK], 64 columns.
    if (tid == 0) {
      fence_after();
      constexpr uint32_t ID = idesc_bf16_mn(128, 64);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t a = sbase + OFF_X + (kk >> 2) * X_ATOM + (kk & 3) * 32;
        mma_bf16(tmem + TM_5, sw128_desc(a), sw128_desc(a), ID, kk > 0 ? 1u : 0u);
      }
    }
    if (!sync_mma()) {
      failed = true;
      break;
    }
    const float gC = gam[63];
    // ---------------------------------------------------------------- phase 1
    if (warp < 2) {  // L = beta_t e^{g_t-g_j} G (j < t) into fp32 shared memory
      const int t = 32 * quarter + lane;
      const float gt = gam[t], bt = betav[t];
#pragma unroll
      for (int c = 0; c < 64; c += 16) {
        float v[16];
        tmem_ld16(tmem + TM_5 + lane_off + c, v);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int j = c + e;
          Lf[t * LDF + j] = j < t ? bt * __expf(gt - gam[j]) * v[e] : 0.f;
        }
      }
    } else if (warp < 4) {  // Mq = e^{g_t-g_j} QK (j <= t), bf16 operand rows 0-63
      const int t = 32 * quarter + lane - 64;
      const float gt = gam[t];
#pragma unroll
      for (int c = 0; c < 64; c += 16) {
        float v[16];
        tmem_ld16(tmem + TM_5 + lane_off + c, v);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int j = c + e;
          v[e] = j <= t ? __expf(gt - gam[j]) * v[e] : 0.f;
        }
        st_chunk(sm + OFF_MQ, swz(t, c), v);
        st_chunk(sm + OFF_MQ, swz(t, c + 8), v + 8);
      }
    }
    fence_proxy();
    fence_before();
    __syncthreads();
    // ---------------------------------------------------------------- phase 2: T = (I + L)^-1
    if (tid < 64) {  // diagonal 16 x 16 blocks by forward substitution, one column per thread
      const int blk = tid >> 4, c = tid & 15, o = 16 * blk;
      float x[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        float acc = r == c ? 1.f : 0.f;
#pragma unroll
        for (int i = 0; i < r; ++i) acc -= Lf[(o + r) * LDF + o + i] * x[i];
        x[r] = acc;
        Tf[(o + r) * LDF + o + c] = acc;
      }
    }
    __syncthreads();
#pragma unroll 1
    for (int d = 1; d < 4; ++d) {  // block (i, j = i - d): T_ij = -T_ii sum_{m=j}^{i-1} L_im T_mj
      const int nb = 4 - d;
      for (int e = tid; e < nb * 256; e += NT) {
        const int j = e >> 8, r = (e >> 4) & 15, c = e & 15, i = j + d;
        float y = 0.f;
        for (int m = j; m < i; ++m) {
#pragma unroll
          for (int x = 0; x < 16; ++x) y += Lf[(16 * i + r) * LDF + 16 * m + x] * Tf[(16 * m + x) * LDF + 16 * j + c];
        }
        Yf[(j * 16 + r) * 17 + c] = y;
      }
      __syncthreads();
      for (int e = tid; e < nb * 256; e += NT) {
        const int j = e >> 8, r = (e >> 4) & 15, c = e & 15, i = j + d;
        float y = 0.f;
#pragma unroll
        for (int x = 0; x < 16; ++x) y += Tf[(16 * i + r) * LDF + 16 * i + x] * Yf[(j * 16 + x) * 17 + c];
        Tf[(16 * i + r) * LDF + 16 * j + c] = -y;
      }
      __syncthreads();
    }
    {  // [T diag(beta b); T diag(beta)] as bf16 operand rows t and 64 + t
      const int t = tid >> 2, j0 = (tid & 3) * 16;
      float w1[16], w2[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int j = j0 + e;
        const float tv = j <= t ? Tf[t * LDF + j] * betav[j] : 0.f;
        w1[e] = tv * bv[j];
        w2[e] = tv;
      }
      st_chunk(sm + OFF_B12, swz(t, j0), w1);
      st_chunk(sm + OFF_B12, swz(t, j0 + 8), w1 + 8);
      st_chunk(sm + OFF_B12, swz(64 + t, j0), w2);
      st_chunk(sm + OFF_B12, swz(64 + t, j0 + 8), w2 + 8);
    }
    fence_proxy();
    fence_before();
    __syncthreads();
    // MMA5: [B1; B2] (K = 64) x [K^T; V^T] (N = 256) -> lanes 0-63: W in columns 0-127, lanes 64-127: U in 128-255.
    if (tid == 0) {
      fence_after();
      constexpr uint32_t ID = idesc_bf16_mn(128, 256);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_bf16(tmem + TM_5, sw128_desc(sbase + OFF_B12 + kk * 32), sw128_desc(sbase + OFF_KVT + kk * 32), ID,
                 kk > 0 ? 1u : 0u);
    }
    if (!sync_mma()) {
      failed = true;
      break;
    }
    // ---------------------------------------------------------------- phase 3: W -> operand rows 128-191
    if (quarter < 2 && (warp == quarter || warp == quarter + 4)) {
      const int t = 32 * quarter + lane, half = warp >> 2;  // half 0: k 0-63, half 1: k 64-127
#pragma unroll
      for (int c = 0; c < 64; c += 16) {
        float v[16];
        tmem_ld16(tmem + TM_5 + lane_off + 64 * half + c, v);
        st_chunk(sm + OFF_X + half * X_ATOM, swz(128 + t, c), v);
        st_chunk(sm + OFF_X + half * X_ATOM, swz(128 + t, c + 8), v + 8);
      }
    }
    fence_proxy();
    fence_before();
    __syncthreads();
    // MMA4: [Q; W] (rows 64-191) x S0^T -> lanes 0-63: Q S0^T, lanes 64-127: W S0^T.
    if (tid == 0) {
      fence_after();
      constexpr uint32_t ID = idesc_bf16_mn(128, 128);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t a = sbase + OFF_X + (kk >> 2) * X_ATOM + 64 * 128 + (kk & 3) * 32;
        const uint32_t bb = sbase + OFF_S + (kk >> 2) * S_ATOM + (kk & 3) * 32;
        mma_bf16(tmem + TM_4, sw128_desc(a), sw128_desc(bb), ID, kk > 0 ? 1u : 0u);
      }
    }
    if (!sync_mma()) {
      failed = true;
      break;
    }
    // ---------------------------------------------------------------- phase 4: D = U - W S0^T, transposed
    if (warp == 4 && ci + 1 < nchunks) gates(ci + 1);  // the next chunk's gates (b_C pre-scales the state)
    if (quarter >= 2 && (warp == quarter || warp == quarter + 4)) {
      const int t = 32 * quarter + lane - 64, half = warp >> 2;  // half: v 0-63 or 64-127
      const float sc = __expf(gC - gam[t]);
#pragma unroll 1
      for (int c = 0; c < 64; c += 16) {
        const int v0 = 64 * half + c;
        float u[16], w[16];
        tmem_ld16(tmem + TM_5 + lane_off + 128 + v0, u);
        tmem_ld16(tmem + TM_4 + lane_off + v0, w);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float dlt = u[e] - w[e];
          st_bf16(sm + OFF_DT, swz(v0 + e, t), dlt);
          st_bf16(sm + OFF_A7, swz(v0 + e, t), dlt * sc);
        }
      }
    }
    fence_proxy();
    fence_before();
    __syncthreads();
    // MMA6: Mq (rows 0-63 meaningful) x D -> TMEM [256, 384);  MMA7: X += A7 x K^T (rows 0-127 of KVT).
    if (tid == 0) {
      fence_after();
      constexpr uint32_t ID = idesc_bf16_mn(128, 128);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_bf16(tmem + TM_5, sw128_desc(sbase + OFF_MQ + kk * 32), sw128_desc(sbase + OFF_DT + kk * 32), ID,
                 kk > 0 ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_bf16(tmem + TM_X, sw128_desc(sbase + OFF_A7 + kk * 32), sw128_desc(sbase + OFF_KVT + kk * 32), ID,
                 (ci > 0 || kk > 0) ? 1u : 0u);
    }
    if (!sync_mma()) {
      failed = true;
      break;
    }
    // ---------------------------------------------------------------- phase 5
    // The staging tiles are dead now: fetch the next chunk's rows behind this phase (warp 7 first
    // completes its z copies of this chunk).
    if (warp == 7) asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (stager && ci + 1 < nchunks) prefetch_rows(ci + 1, stage_idx);
    // O = b_t Q S0^T + Mq D with the gated RMSNorm: rows t = TMEM lanes 0-63 (warps 0, 1, 4, 5; each
    // warp owns 64 of the 128 columns).  Every lane runs the warp-collective TMEM loads; rows t < n are stored.
    const int half = warp >> 2;
    if (quarter < 2) {
      const int t = 32 * quarter + lane;
      const float bt = bv[t];
      float ss = 0.f;
#pragma unroll 1
      for (int c = 64 * half; c < 64 * half + 64; c += 16) {
        float a[16], d[16];
        tmem_ld16(tmem + TM_4 + lane_off + c, a);
        tmem_ld16(tmem + TM_5 + lane_off + c, d);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float o = bt * a[e] + d[e];
          ss += o * o;
        }
      }
      part[half * 64 + t] = ss;
    }
    __syncthreads();
    if (quarter < 2) {
      const int t = 32 * quarter + lane;
      const float bt = bv[t];
      const float inv = rsqrtf((part[t] + part[64 + t]) / K + p.eps);
      __nv_bfloat16* dst = p.out + (t0 + c0 + min(t, n - 1)) * p.out_stride + hv * K;
      const uint8_t* zrow = sm + OFF_Z + t * 256;
#pragma unroll 1
      for (int c = 64 * half; c < 64 * half + 64; c += 16) {
        float a[16], d[16], o[16];
        tmem_ld16(tmem + TM_4 + lane_off + c, a);
        tmem_ld16(tmem + TM_5 + lane_off + c, d);
        const uint4 z0 = *reinterpret_cast<const uint4*>(zrow + ((((c >> 3)) ^ (t & 7)) << 4));
        const uint4 z1 = *reinterpret_cast<const uint4*>(zrow + ((((c >> 3) + 1) ^ (t & 7)) << 4));
        const uint32_t zw[8] = {z0.x, z0.y, z0.z, z0.w, z1.x, z1.y, z1.z, z1.w};
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float zv = (e & 1) ? hi(zw[e >> 1]) : lo(zw[e >> 1]);
          o[e] = (bt * a[e] + d[e]) * inv * nw[c + e] * silu(zv);
        }
        if (t < n) {
          uint4 u0, u1;
          u0.x = pack_bf16(o[0], o[1]);
          u0.y = pack_bf16(o[2], o[3]);
          u0.z = pack_bf16(o[4], o[5]);
          u0.w = pack_bf16(o[6], o[7]);
          u1.x = pack_bf16(o[8], o[9]);
          u1.y = pack_bf16(o[10], o[11]);
          u1.z = pack_bf16(o[12], o[13]);
          u1.w = pack_bf16(o[14], o[15]);
          reinterpret_cast<uint4*>(dst + c)[0] = u0;
          reinterpret_cast<uint4*>(dst + c)[1] = u1;
        }
      }
    }
    {  // state rows v = TMEM lanes (all warps, 64 columns each): bf16 S0 of the next chunk and the state
       // pre-scaled by the next chunk's total decay b_C (the S_C = b_C S0 + ... term); fp32 to global after
       // the last chunk
      const int v = 32 * quarter + lane;
      const bool last = ci == nchunks - 1;
      const float bnext = last ? 1.f : bv_all[((ci + 1) & 1) * 64 + 63];
      float* srow = p.state + ((slot * p.HV + hv) * K + v) * K;
#pragma unroll 1
      for (int c = 64 * half; c < 64 * half + 64; c += 16) {
        float x[16];
        tmem_ld16(tmem + TM_X + lane_off + c, x);
        st_chunk(sm + OFF_S + half * S_ATOM, swz(v, c & 63), x);
        st_chunk(sm + OFF_S + half * S_ATOM, swz(v, (c & 63) + 8), x + 8);
        if (last) {
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4*>(srow + c + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) x[e] *= bnext;
          tmem_st16(tmem + TM_X + lane_off + c, x);
        }
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    if (stager) asm volatile("cp.async.wait_group 0;" ::: "memory");  // the next chunk's rows have landed
    fence_proxy();
    fence_before();
    __syncthreads();
  }
  if (failed) {
    if (p.err) atomicExch(p.err, 1);
    if (tid == 0) mbar_wait_drain(bar, phase ^ 1);  // the group whose wait gave up
  } else if (nchunks == 0) {  // empty request: the committed state is zero
    for (int i = tid; i < K * K; i += NT) p.state[(slot * p.HV + hv) * K * K + i] = 0.f;
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS));
  }
}

}  // namespace gdnc
}  // namespace shk

extern "C" int sh_gdn_chunk_prefill(const GdnParams* p, int batch, cudaStream_t stream) {
  using namespace shk::gdnc;
  if (batch <= 0) return 0;
  if (p->K != K || p->V != K || p->HV % p->H != 0) return -1;
  auto al16 = [](const void* ptr, int64_t stride) {
    return reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && (stride * 2) % 16 == 0;
  };
  if (!al16(p->qkv, p->qkv_stride) || !al16(p->z, p->z_stride) || !al16(p->out, p->out_stride)) return -3;
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(gdn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr = true;
  }
  shk::launch(gdn_chunk_kernel, dim3(batch, p->HV), dim3(NT), SMEM_ALLOC, stream, *p);
  return static_cast<int>(cudaGetLastError());
}
