// Multi-head latent attention (DeepSeek-V3 / Kimi-K2 absorbed form) decode and
// the DeepSeek-V3.2 lightning indexer with top-k selection.
//
// MLA decode.  Queries are already absorbed into the latent space: q[t, h] =
// [q_nope W_UK | rotated q_pe] (C = kv_lora + rope columns); the paged cache
// row of a key is [normalised c_kv | rotated k_pe], and the values are the
// first V = kv_lora columns of the same row.  Work unit = (query token, 64
// heads, key split): all heads of a token share every key, so a 32-key
// sub-page gathered once feeds 64 rows of bf16 tensor-core tiles (mma.sync
// m16n8k16, fp32 accumulate).  8 warps = 4 row groups (16 heads) x 2 halves:
// for QK^T the two warps of a row group take one half of the 32 keys each
// (C-deep dot products), exchange row maxima and their probabilities P
// through shared memory, and for PV each takes one half of the V columns over
// all 32 keys, so the [16 x V/2] fp32 accumulator of a warp stays in
// registers.  Keys come from a DSA top-k list (sparse) or every position up to
// the token's own (dense causal); a key position outside the causal range or
// -1 is zero-filled and masked.  Sub-pages are gathered row by row with
// cp.async (two-stage ring), which serves both the contiguous and the sparse
// case.  Online softmax in the exp2 domain; with nsplit > 1 each split writes
// normalised O and (max, sum) and mla_merge combines them in split order.
//
// DSA indexer.  logits[t, s] = sum_h relu(q[t, h] . k[s]) * w[t, h] over the
// token's causal keys, computed on tensor-core tiles (16 heads x 64 keys per
// warp), then the top K positions by a 4-pass radix select on the float
// bits; ties at the threshold keep the latest positions, and the selected
// positions are written in ascending order (a deterministic key order for the
// attention that follows).
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "mla.h"
#include "pdl.cuh"

namespace shk {
namespace mla {

constexpr int ROWS = 64;  // heads per work unit
constexpr int KEYS = 32;  // keys per sub-page
constexpr int THREADS = 256;
constexpr int P_LD = 40;  // bf16 row stride of the P tile (80 bytes)

__device__ __forceinline__ uint32_t saddr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0));
}
__device__ __forceinline__ void ldsm_x4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// [NR rows][C] bf16 tile as C/64 slabs of [NR][128 B]; 16-byte chunk cc of row
// r sits at chunk position cc ^ (r & 7) of its slab (conflict-free ldmatrix).
template <int NR>
__device__ __forceinline__ uint32_t swz(int r, int cc) {
  return static_cast<uint32_t>((cc >> 3) * (NR * 128) + r * 128 + (((cc & 7) ^ (r & 7)) << 4));
}
// Request of query token t: the largest b with q_start[b] <= t.
__device__ __forceinline__ int request_of(const int64_t* q_start, int B, int t) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (q_start[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}
__device__ __forceinline__ void bar_pair(int id) { asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory"); }

// NVFP4 row (mla.h): e2m1 pairs, R e4m3 rope bytes, Cl/16 permuted e4m3 block scales, padded to 16 bytes.
__host__ __device__ constexpr int fp4_rope_off(int Cl) { return Cl / 2; }
__host__ __device__ constexpr int fp4_sc_off(int Cl, int R) { return Cl / 2 + R; }
__host__ __device__ constexpr int fp4_sc_pos(int Cl, int s) { return (Cl / 64) * (s & 3) + (s >> 2); }
__host__ __device__ constexpr int fp4_row_bytes(int Cl, int R) { return (Cl / 2 + R + Cl / 16 + 15) / 16 * 16; }

template <int C, int V, bool FP4>
struct MlaSmem {
  static constexpr int Q_BYTES = ROWS * C * 2;
  static constexpr int KV_BYTES = KEYS * C * 2;
  static constexpr int ROWB = fp4_row_bytes(V, C - V);
  static constexpr int RAW_BYTES = FP4 ? KEYS * ROWB : 0;  // packed rows of one sub-page (NVFP4 cache)
  static constexpr int RAW_OFF = Q_BYTES + 2 * KV_BYTES;
  static constexpr int P_OFF = RAW_OFF + 2 * RAW_BYTES;
  static constexpr int M_OFF = P_OFF + 4 * 16 * P_LD * 2;
  static constexpr int L_OFF = M_OFF + 4 * 2 * 16 * 4;
  static constexpr int I_OFF = L_OFF + 4 * 2 * 16 * 4;  // [3][KEYS] physical cache rows (-1: masked key)
  static constexpr int TOTAL = I_OFF + 3 * KEYS * 8 + 128;
  static_assert(TOTAL <= 227 * 1024, "shared memory budget");
};

// e2m1 code (bits 0-3) times the e4m3 scale, as bf16 (exact: at most 6 significant bits).  The code's bits
// placed at bf16 positions 15 / 6..8 read as code_value * 2^-126 (fp32 upper half); two power-of-two
// multiplies restore the scale without overflow.
__device__ __forceinline__ float fp4_value(uint32_t code, float scale_x2p63) {
  const uint32_t bits = ((code & 7u) << 22) | ((code & 8u) << 28);
  return (__uint_as_float(bits) * 9.223372036854775808e18f) * scale_x2p63;
}

template <int C, int V, bool FP4>
__global__ void __launch_bounds__(THREADS, 1) mla_decode_kernel(MlaParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  using S = MlaSmem<C, V, FP4>;
  constexpr int CH = C / 8;        // 16-byte chunks per row
  constexpr int KSTEPS = C / 16;
  constexpr int VH = V / 2;        // value columns per warp
  constexpr int VT = VH / 8;       // n8 tiles per warp
  static_assert(C % 64 == 0 && V % 32 == 0 && V <= C, "MLA geometry");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const uint32_t sQ = saddr(smem);
  const uint32_t sKV = sQ + S::Q_BYTES;
  __nv_bfloat16* sP = reinterpret_cast<__nv_bfloat16*>(smem + S::P_OFF);
  float* sM = reinterpret_cast<float*>(smem + S::M_OFF);
  float* sL = reinterpret_cast<float*>(smem + S::L_OFF);
  int64_t* sRow = reinterpret_cast<int64_t*>(smem + S::I_OFF);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rg = warp & 3, vh = warp >> 2, g = lane >> 2, t4 = lane & 3;
  const int t = blockIdx.x, h0 = blockIdx.y * ROWS, split = blockIdx.z;
  const int b = request_of(p.q_start, p.B, t);
  const int64_t qs = p.q_start[b], ql = p.q_start[b + 1] - qs, seq = p.seq_lens[b];
  const int64_t qpos = seq - ql + (t - qs);
  const int64_t nkeys = p.topk ? static_cast<int64_t>(p.topk_k) : qpos + 1;
  const int npages = static_cast<int>((nkeys + KEYS - 1) / KEYS);
  const int per = (npages + p.nsplit - 1) / p.nsplit;
  const int pg0 = min(split * per, npages), pg1 = min(pg0 + per, npages);
  const int rows_valid = min(ROWS, p.H - h0);
  const int32_t* bt = p.block_tables + static_cast<int64_t>(b) * p.bt_stride;

  // Key position of entry `key` of sub-page j (-1: past the list, unused or outside the causal range).
  auto key_pos = [&](int j, int key) -> int64_t {
    const int64_t kp = static_cast<int64_t>(j) * KEYS + key;
    if (j >= pg1 || kp >= nkeys) return -1;
    const int64_t pos = p.topk ? static_cast<int64_t>(p.topk[static_cast<int64_t>(t) * p.topk_k + kp]) : kp;
    return (pos < 0 || pos > qpos) ? -1 : pos;
  };
  auto row_of = [&](int64_t pos) -> int64_t {
    return pos < 0 ? -1 : static_cast<int64_t>(bt[pos >> 6]) * 64 + (pos & 63);
  };
  // Issue the cp.async gather of sub-page j (rows already in sRow[j % 3]) into stage st (NVFP4: the packed
  // rows go to the raw ring and are decoded into the stage by `decode_page`).
  const uint32_t sRaw = sQ + S::RAW_OFF;
  auto load_page = [&](int j, int st) {
    const int64_t* rows = sRow + (j % 3) * KEYS;
    if constexpr (FP4) {
      constexpr int RCH = S::ROWB / 16;
      for (int c = tid; c < KEYS * RCH; c += THREADS) {
        const int key = c / RCH, cc = c % RCH;
        const int64_t row = rows[key];
        cp_async16(sRaw + st * S::RAW_BYTES + key * S::ROWB + cc * 16,
                   p.latent_fp4 + (row < 0 ? 0 : row) * S::ROWB + cc * 16, row >= 0);
      }
    } else {
      for (int c = tid; c < KEYS * CH; c += THREADS) {
        const int key = c / CH, cc = c % CH;
        const int64_t row = rows[key];
        cp_async16(sKV + st * S::KV_BYTES + swz<KEYS>(key, cc), p.latent + (row < 0 ? 0 : row) * C + cc * 8,
                   row >= 0);
      }
    }
  };
  // NVFP4: packed latent blocks -> bf16 chunks of the swizzled stage; rope chunks copied as they are.
  auto decode_page = [&](int st) {
    constexpr int NB = V / 16;
    const uint8_t* raw = smem + S::RAW_OFF + st * S::RAW_BYTES;
    uint8_t* kvp = smem + S::Q_BYTES + st * S::KV_BYTES;
    for (int i = tid; i < KEYS * NB; i += THREADS) {
      const int key = i / NB, blk = i % NB;
      const uint8_t* r = raw + key * S::ROWB;
      const uint2 pk = *reinterpret_cast<const uint2*>(r + blk * 8);
      __nv_fp8_e4m3 s8;
      s8.__x = r[fp4_sc_off(V, C - V) + fp4_sc_pos(V, blk)];
      const float sc = static_cast<float>(s8) * 9.223372036854775808e18f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t w = h ? pk.y : pk.x;
        uint32_t outw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t byte = (w >> (8 * e)) & 0xFFu;
          outw[e] = pack2(fp4_value(byte & 15u, sc), fp4_value(byte >> 4, sc));
        }
        *reinterpret_cast<uint4*>(kvp + swz<KEYS>(key, blk * 2 + h)) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
      }
    }
    constexpr int RC = (C - V) / 8;  // 16-byte bf16 chunks of the rope, 8 e4m3 bytes each
    for (int i = tid; i < KEYS * RC; i += THREADS) {
      const int key = i / RC, rc = i % RC;
      uint32_t w[4];
      e4m3x8_to_bf16(*reinterpret_cast<const uint2*>(raw + key * S::ROWB + fp4_rope_off(V) + rc * 8), w);
      *reinterpret_cast<uint4*>(kvp + swz<KEYS>(key, V / 8 + rc)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  };

  if (warp == 0) {  // rows of the first two sub-pages
    sRow[(pg0 % 3) * KEYS + lane] = row_of(key_pos(pg0, lane));
    sRow[((pg0 + 1) % 3) * KEYS + lane] = row_of(key_pos(pg0 + 1, lane));
  }
  for (int c = tid; c < ROWS * CH; c += THREADS) {
    const int r = c / CH, cc = c % CH;
    const bool ok = r < rows_valid;
    cp_async16(sQ + swz<ROWS>(r, cc), p.q + (static_cast<int64_t>(t) * p.H + h0 + (ok ? r : 0)) * C + cc * 8, ok);
  }
  asm volatile("cp.async.commit_group;\n" ::);
  __syncthreads();
  if (pg0 < pg1) load_page(pg0, 0);
  asm volatile("cp.async.commit_group;\n" ::);

  float o[VT][4];
#pragma unroll
  for (int i = 0; i < VT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  __nv_bfloat16* myP = sP + rg * 16 * P_LD;
  const uint32_t sPrg = saddr(myP);

  for (int j = pg0; j < pg1; ++j) {
    const int st = (j - pg0) & 1;
    if (j + 1 < pg1) load_page(j + 1, st ^ 1);
    asm volatile("cp.async.commit_group;\n" ::);
    // warp 0 fetches sub-page j+2's positions now and resolves its rows after the QK^T below,
    // so both dependent global loads overlap this sub-page's tensor-core work
    int64_t nxt_pos = -1;
    if (warp == 0) nxt_pos = key_pos(j + 2, lane);
    asm volatile("cp.async.wait_group 1;\n" ::);
    __syncthreads();
    if constexpr (FP4) {
      decode_page(st);
      __syncthreads();
    }
    const uint32_t kv = sKV + st * S::KV_BYTES;
    const int64_t* rows_j = sRow + (j % 3) * KEYS;
    // S = Q K^T for this warp's 16 heads x 16 keys (even and odd k-steps accumulate apart: 4 chains)
    float sc[2][4], sd[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = sd[i][0] = sd[i][1] = sd[i][2] = sd[i][3] = 0.f;
#pragma unroll 4
    for (int kk = 0; kk < KSTEPS; kk += 2) {
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
      ldsm_x4(sQ + swz<ROWS>(rg * 16 + (lane & 15), 2 * kk + (lane >> 4)), a0, a1, a2, a3);
      ldsm_x4(kv + swz<KEYS>(vh * 16 + (lane & 7) + ((lane >> 4) << 3), 2 * kk + ((lane >> 3) & 1)), b0, b1, b2, b3);
      mma16816(sc[0], a0, a1, a2, a3, b0, b1);
      mma16816(sc[1], a0, a1, a2, a3, b2, b3);
      ldsm_x4(sQ + swz<ROWS>(rg * 16 + (lane & 15), 2 * (kk + 1) + (lane >> 4)), a0, a1, a2, a3);
      ldsm_x4(kv + swz<KEYS>(vh * 16 + (lane & 7) + ((lane >> 4) << 3), 2 * (kk + 1) + ((lane >> 3) & 1)), b0, b1, b2,
              b3);
      mma16816(sd[0], a0, a1, a2, a3, b0, b1);
      mma16816(sd[1], a0, a1, a2, a3, b2, b3);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[i][e] += sd[i][e];
    if (warp == 0) {
      const int64_t r = row_of(nxt_pos);
      sRow[((j + 2) % 3) * KEYS + lane] = r;  // read by load_page(j + 2) after the next __syncthreads
    }
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool valid = rows_j[vh * 16 + nt * 8 + 2 * t4 + e] >= 0;
        const float va = valid ? sc[nt][e] * p.scale_log2 : -INFINITY;
        const float vb = valid ? sc[nt][2 + e] * p.scale_log2 : -INFINITY;
        sc[nt][e] = va;
        sc[nt][2 + e] = vb;
        mx_a = fmaxf(mx_a, va);
        mx_b = fmaxf(mx_b, vb);
      }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    if (t4 == 0) {
      sM[(rg * 2 + vh) * 16 + g] = mx_a;
      sM[(rg * 2 + vh) * 16 + g + 8] = mx_b;
    }
    bar_pair(1 + rg);
    mx_a = fmaxf(mx_a, sM[(rg * 2 + (vh ^ 1)) * 16 + g]);
    mx_b = fmaxf(mx_b, sM[(rg * 2 + (vh ^ 1)) * 16 + g + 8]);
    const float nm_a = fmaxf(m_a, mx_a), nm_b = fmaxf(m_b, mx_b);
    const float base_a = nm_a == -INFINITY ? 0.f : nm_a, base_b = nm_b == -INFINITY ? 0.f : nm_b;
    const float al_a = exp2f(m_a - base_a), al_b = exp2f(m_b - base_b);
    float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const float p0 = exp2f(sc[nt][0] - base_a), p1 = exp2f(sc[nt][1] - base_a);
      const float p2 = exp2f(sc[nt][2] - base_b), p3 = exp2f(sc[nt][3] - base_b);
      sum_a += p0 + p1;
      sum_b += p2 + p3;
      const int col = vh * 16 + nt * 8 + 2 * t4;
      *reinterpret_cast<uint32_t*>(myP + g * P_LD + col) = pack2(p0, p1);
      *reinterpret_cast<uint32_t*>(myP + (g + 8) * P_LD + col) = pack2(p2, p3);
    }
    l_a = l_a * al_a + sum_a;  // this warp's keys; the two halves are added at the end
    l_b = l_b * al_b + sum_b;
    m_a = nm_a;
    m_b = nm_b;
#pragma unroll
    for (int dt = 0; dt < VT; ++dt) {
      o[dt][0] *= al_a;
      o[dt][1] *= al_a;
      o[dt][2] *= al_b;
      o[dt][3] *= al_b;
    }
    bar_pair(1 + rg);  // both halves of P are written
    // O[16 x V/2] += P[16 x 32] V[32 x V/2]
#pragma unroll
    for (int kc = 0; kc < 2; ++kc) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(sPrg + ((lane & 15) * P_LD + kc * 16 + (lane >> 4) * 8) * 2, a0, a1, a2, a3);
#pragma unroll
      for (int dp = 0; dp < VT / 2; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(kv + swz<KEYS>(kc * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), vh * (VH / 8) + 2 * dp + (lane >> 4)),
                  b0, b1, b2, b3);
        mma16816(o[2 * dp], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // stage st, P and the maxima are free for the next sub-page
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  if (t4 == 0) {
    sL[(rg * 2 + vh) * 16 + g] = l_a;
    sL[(rg * 2 + vh) * 16 + g + 8] = l_b;
  }
  bar_pair(1 + rg);
  l_a += sL[(rg * 2 + (vh ^ 1)) * 16 + g];
  l_b += sL[(rg * 2 + (vh ^ 1)) * 16 + g + 8];
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f, inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = rg * 16 + g + 8 * half;
    if (r >= rows_valid) continue;
    const int64_t th = static_cast<int64_t>(t) * p.H + h0 + r;
    const float inv = half ? inv_b : inv_a;
    if (p.nsplit == 1) {
      __nv_bfloat16* dst = p.out + th * V + vh * VH;
#pragma unroll
      for (int dt = 0; dt < VT; ++dt)
        *reinterpret_cast<__nv_bfloat162*>(dst + dt * 8 + 2 * t4) =
            __floats2bfloat162_rn(o[dt][2 * half] * inv, o[dt][2 * half + 1] * inv);
    } else {
      const int64_t prow = th * p.nsplit + split;
      float* dst = p.part_o + prow * V + vh * VH;
#pragma unroll
      for (int dt = 0; dt < VT; ++dt)
        *reinterpret_cast<float2*>(dst + dt * 8 + 2 * t4) = make_float2(o[dt][2 * half] * inv, o[dt][2 * half + 1] * inv);
      if (t4 == 0 && vh == 0) {
        p.part_ml[prow * 2] = half ? m_b : m_a;
        p.part_ml[prow * 2 + 1] = half ? l_b : l_a;
      }
    }
  }
}

// out[t, h, :] = sum_s w_s o_s / sum_s w_s, w_s = l_s exp2(m_s - max m), in split order.
__global__ void mla_merge_kernel(__nv_bfloat16* __restrict__ out, const float* __restrict__ part_o,
                                 const float* __restrict__ part_ml, int64_t rows, int nsplit, int V) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int per_row = V / 2;
  if (i >= rows * per_row) return;
  const int64_t row = i / per_row;
  const int c = static_cast<int>(i % per_row) * 2;
  float mx = -INFINITY;
  for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, part_ml[(row * nsplit + s) * 2]);
  const float base = mx == -INFINITY ? 0.f : mx;
  float acc0 = 0.f, acc1 = 0.f, den = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const int64_t pr = row * nsplit + s;
    const float w = part_ml[pr * 2 + 1] * exp2f(part_ml[pr * 2] - base);
    const float2 v = *reinterpret_cast<const float2*>(part_o + pr * V + c);
    acc0 += w * v.x;
    acc1 += w * v.y;
    den += w;
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  *reinterpret_cast<__nv_bfloat162*>(out + row * V + c) = __floats2bfloat162_rn(acc0 * inv, acc1 * inv);
}

__global__ void cache_write_kernel(__nv_bfloat16* __restrict__ latent, const __nv_bfloat16* __restrict__ c,
                                   int64_t c_stride, const __nv_bfloat16* __restrict__ kpe, int64_t kpe_stride,
                                   const int64_t* __restrict__ slots, int Cl, int R) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int t = blockIdx.x;
  const int64_t slot = slots[t];
  if (slot < 0) return;
  __nv_bfloat16* dst = latent + slot * (Cl + R);
  for (int i = threadIdx.x; i < Cl + R; i += blockDim.x)
    dst[i] = i < Cl ? c[t * c_stride + i] : kpe[t * kpe_stride + (i - Cl)];
}

// NVFP4 latent row writer (layout: sh_mla_fp4_row_bytes): one CTA of 64 threads per token; thread i
// quantises latent block i (16 values) and the threads round the rope values to e4m3.
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

__global__ void cache_write_fp4_kernel(uint8_t* __restrict__ cache, const __nv_bfloat16* __restrict__ c,
                                       int64_t c_stride, const __nv_bfloat16* __restrict__ kpe, int64_t kpe_stride,
                                       const int64_t* __restrict__ slots, int Cl, int R) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int t = blockIdx.x;
  const int64_t slot = slots[t];
  if (slot < 0) return;
  uint8_t* row = cache + slot * fp4_row_bytes(Cl, R);
  const int blk = threadIdx.x;
  if (blk < Cl / 16) {
    float v[16];
    float am = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[j] = __bfloat162float(c[t * c_stride + blk * 16 + j]);
      am = fmaxf(am, fabsf(v[j]));
    }
    // round to nearest even, saturating; the 2^-9 floor (the smallest e4m3 subnormal) keeps the scale nonzero
    const __nv_fp8_e4m3 s(fmaxf(__fdiv_rn(am, 6.f), 1.953125e-3f));
    const float inv = __frcp_rn(static_cast<float>(s));  // correctly rounded, as the CPU statement
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] *= inv;
    *reinterpret_cast<uint2*>(row + blk * 8) = make_uint2(e2m1x8(v), e2m1x8(v + 8));
    row[fp4_sc_off(Cl, R) + fp4_sc_pos(Cl, blk)] = s.__x;
  }
  for (int i = threadIdx.x; i < R; i += blockDim.x)
    row[fp4_rope_off(Cl) + i] = __nv_fp8_e4m3(__bfloat162float(kpe[t * kpe_stride + i])).__x;
}

}  // namespace mla
}  // namespace shk

using namespace shk::mla;

namespace {
template <int C, int V, bool FP4>
int launch_mla(const MlaParams& p, cudaStream_t st) {
  using S = MlaSmem<C, V, FP4>;
  auto k = mla_decode_kernel<C, V, FP4>;
  static bool ready = false;
  if (!ready) {
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL);
    if (e != cudaSuccess) return static_cast<int>(e);
    ready = true;
  }
  int r = -2;
  if constexpr (C == 576 && V == 512)
    if (p.impl != 1) r = sh_mla_decode_tc(&p, st);  // -2: the tcgen05 kernel does not apply
  if (r == -2) {
    shk::launch(k, dim3(p.T, (p.H + ROWS - 1) / ROWS, p.nsplit), dim3(THREADS), S::TOTAL, st, p);
    r = static_cast<int>(cudaGetLastError());
  }
  if (r || p.nsplit == 1) return r;
  const int64_t rows = static_cast<int64_t>(p.T) * p.H;
  const int64_t n = rows * (V / 2);
  shk::launch(mla_merge_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, st, p.out, p.part_o,
              p.part_ml, rows, p.nsplit, V);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

extern "C" int sh_mla_decode(const MlaParams* p, int C, int V, cudaStream_t stream) {
  if (p->T <= 0) return 0;
  if (p->nsplit < 1 || (p->nsplit > 1 && (!p->part_o || !p->part_ml))) return -1;
  const bool fp4 = p->latent_fp4 != nullptr;
  if (C == 576 && V == 512) return fp4 ? launch_mla<576, 512, true>(*p, stream) : launch_mla<576, 512, false>(*p, stream);
  if (C == 128 && V == 64) return fp4 ? launch_mla<128, 64, true>(*p, stream) : launch_mla<128, 64, false>(*p, stream);
  return -2;
}

extern "C" int sh_mla_fp4_row_bytes(int Cl, int R) { return fp4_row_bytes(Cl, R); }

extern "C" int sh_mla_cache_write_fp4(uint8_t* cache, const __nv_bfloat16* c, int64_t c_stride,
                                      const __nv_bfloat16* kpe, int64_t kpe_stride, const int64_t* slots, int T,
                                      int Cl, int R, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (Cl % 64 != 0 || Cl / 16 > 64) return -2;
  shk::launch(cache_write_fp4_kernel, dim3(T), dim3(64), 0, stream, cache, c, c_stride, kpe, kpe_stride, slots, Cl,
              R);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_mla_cache_write(__nv_bfloat16* latent, const __nv_bfloat16* c, int64_t c_stride,
                                  const __nv_bfloat16* kpe, int64_t kpe_stride, const int64_t* slots, int T, int Cl,
                                  int R, cudaStream_t stream) {
  if (T <= 0) return 0;
  shk::launch(cache_write_kernel, dim3(T), dim3(128), 0, stream, latent, c, c_stride, kpe, kpe_stride, slots, Cl, R);
  return static_cast<int>(cudaGetLastError());
}

