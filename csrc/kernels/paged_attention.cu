// Paged GQA attention for prefill, decode and speculative verify.
//
// Work unit = (64-row query tile, kv head, kv split).  A query tile packs
// (token, q-head-of-this-group) rows: row r -> token r / G, head h*G + r % G,
// so the G query heads sharing a kv head and the k+1 verify tokens of a
// request read every K/V page once per split.  Each request's pages are cut
// into `nsplit` equal chunks (split-KV) so short batches still fill the SMs;
// with nsplit > 1 every unit writes an fp32 partial (normalised O, row max,
// row sum) to a workspace and attn_merge combines them in split order.
//
// Per CTA: warp 0 is a TMA producer streaming 64-token K and V pages of the
// [num_blocks, kv_heads, 64, D] cache (viewed as 2-D rows of D) in 128-byte
// swizzled 64-column boxes into a 4-stage mbarrier ring; warps 1..4 each own
// 16 query rows and run QK^T / PV on bf16 tensor-core tiles (mma.sync
// m16n8k16, fp32 accumulate) with an exp2 online softmax.  Causality is by
// absolute position: the query token at position p sees keys [0, p].  Every
// mbarrier wait is bounded and reports a timeout through *err.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <mutex>

#include "paged_attention.h"
#include "pdl.cuh"

namespace shk {
namespace attn {

constexpr int ROWS = 64;   // query rows per unit
constexpr int KEYS = 64;   // keys per page
constexpr int THREADS = 160;
constexpr uint64_t kTimeoutNs = 2000000000ull;

__device__ __forceinline__ uint32_t saddr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t c) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(c));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t par) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(par)
      : "memory");
  return ok != 0;
}
// try_wait that may suspend the thread in hardware (up to hint_ns) until the phase completes.
__device__ __forceinline__ bool mbar_try_sleep(uint64_t* b, uint32_t par, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(par), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t par, volatile int* abort_flag) {
  if (mbar_try(b, par)) return true;
  const uint64_t t0 = now_ns();
  while (true) {  // poll without a suspend hint (a suspended warp can wake up late); checks every 64 polls
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try(b, par)) return true;
    if (*abort_flag) return false;
    if (now_ns() - t0 > kTimeoutNs) return false;
  }
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* m, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          saddr(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(saddr(bar))
      : "memory");
}
__device__ __forceinline__ void cp_async16(void* smem, const void* g, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr(smem)), "l"(g), "r"(pred ? 16 : 0));
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

// A [64 rows][D] bf16 tile stored as D/64 column slabs of [64 rows][128 B],
// each slab in the TMA 128-byte swizzle: 16-byte chunk c of row r sits at
// chunk position c ^ (r & 7).  `cc` is the logical 16-byte chunk (0..D/8-1).
__device__ __forceinline__ uint32_t swz(int r, int cc) {
  return static_cast<uint32_t>((cc >> 3) * (64 * 128) + r * 128 + (((cc & 7) ^ (r & 7)) << 4));
}

// K/V page ring depth: as deep as the 227 KB block budget allows (the key-split
// variants also hold the merge area), so more page bytes are in flight per SM.
template <int D, int KS>
struct Stages {
  static constexpr int value = D == 64 ? 8 : (D == 128 ? (KS > 1 ? 5 : 6) : 2);
};

// Geometry of one work unit, computed identically by the producer and the
// compute warps.
struct Unit {
  int b, row0, h, split;
  int64_t qs, seq_len, ctx0;
  int q_len, rows_valid, pg0, pg1;
};

__device__ __forceinline__ Unit unit_of(const AttnParams& p, int u, int ntiles) {
  Unit w;
  const int per_tile = p.hk * p.nsplit;
  const int tile = u / per_tile;
  const int rem = u % per_tile;
  w.h = rem / p.nsplit;
  w.split = rem % p.nsplit;
  w.b = p.tile_req[tile];
  w.row0 = p.tile_row0[tile];
  const int G = p.hq / p.hk;
  w.qs = p.q_start[w.b];
  w.q_len = static_cast<int>(p.q_start[w.b + 1] - w.qs);
  w.seq_len = p.seq_lens[w.b];
  w.ctx0 = w.seq_len - w.q_len;
  w.rows_valid = min(ROWS, w.q_len * G - w.row0);
  const int64_t kv_end = min(w.seq_len, w.ctx0 + (w.row0 + w.rows_valid - 1) / G + 1);
  const int npages = static_cast<int>((kv_end + KEYS - 1) / KEYS);
  const int per = (npages + p.nsplit - 1) / p.nsplit;
  w.pg0 = min(w.split * per, npages);
  w.pg1 = min(w.pg0 + per, npages);
  return w;
}

// Persistent: gridDim.x CTAs loop over units u = blockIdx.x + i * gridDim.x;
// the producer's page ring runs continuously across unit boundaries.
template <int D, int KS>
__global__ void __launch_bounds__(THREADS, 1)
    paged_attn_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, AttnParams p,
                      int ntiles) {
  constexpr int TILE_BYTES = 64 * D * 2;  // one [64][D] bf16 tile
  constexpr int STAGES = Stages<D, KS>::value;
  constexpr int KSTEPS = D / 16;
  constexpr int DT = D / 8;
  constexpr int NT = 8 / KS;  // 8-key n-tiles per page per warp
  constexpr int KC = 4 / KS;  // 16-key PV chunks per page per warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + TILE_BYTES;  // stage s: K at s*2*TILE, V at s*2*TILE + TILE
  float* sMerge = reinterpret_cast<float*>(sKV + STAGES * 2 * TILE_BYTES);  // [4 warps][32][DT*4+4]
  uint64_t* full = reinterpret_cast<uint64_t*>(sMerge + (KS > 1 ? 4 * 32 * (DT * 4 + 4) : 0));
  uint64_t* empty = full + STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + STAGES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.hq / p.hk;
  const int units = ntiles * p.hk * p.nsplit;
  if (threadIdx.x == 0) {
    // fetch the tensor-map descriptors while the barriers are set up
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmK)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmV)) : "memory");
    for (int st = 0; st < STAGES; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], 4);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // Dependents may launch once this CTA works on its last unit (triggered below), not at its start:
  // their CTAs would otherwise sit on the SMs for the whole kernel.
  if (blockIdx.x >= units) shk::pdl_trigger();
  shk::pdl_wait();  // inputs of the previous kernel are complete from here on

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int issued = 0;
      bool aborted = false;
      for (int u = blockIdx.x; u < units && !aborted; u += gridDim.x) {
        const Unit w = unit_of(p, u, ntiles);
        const int32_t* bt = p.block_tables + static_cast<int64_t>(w.b) * p.bt_stride;
        for (int j = w.pg0; j < w.pg1; ++j, ++issued) {
          const int st = issued % STAGES;
          if (!mbar_wait(&empty[st], ((issued / STAGES) & 1) ^ 1, abort_flag)) {
            if (p.err) atomicCAS(p.err, 0, 11);
            *abort_flag = 1;
            aborted = true;
            break;
          }
          const int y = (bt[j] * p.hk + w.h) * KEYS;
          uint8_t* dk = sKV + st * 2 * TILE_BYTES;
          mbar_expect_tx(&full[st], 2 * TILE_BYTES);
#pragma unroll
          for (int slab = 0; slab < D / 64; ++slab) {
            tma_2d(dk + slab * 64 * 128, &tmK, slab * 64, y, &full[st]);
            tma_2d(dk + TILE_BYTES + slab * 64 * 128, &tmV, slab * 64, y, &full[st]);
          }
        }
      }
      if (aborted) {  // let every issued load land before exit (bounded)
        for (int i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i) {
          const uint64_t t0 = now_ns();
          while (!mbar_try(&full[i % STAGES], (i / STAGES) & 1))
            if (now_ns() - t0 > kTimeoutNs) break;
        }
      }
    }
    return;
  }
  // -------------------------------------------------------------- compute
  // Warp cw owns row block cw / KS (16 rows) and key part cw % KS (64 / KS
  // keys of every page); the KS partial softmax states of a row block are
  // merged through shared memory at the end of each unit.
  const int cw = warp - 1;
  const int rbk = cw / KS, kpart = cw % KS;
  const int g = lane >> 2, t4 = lane & 3;
  const int key0 = kpart * (KEYS / KS);
  int it = 0;  // pages consumed by this CTA so far (ring position)
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    if (u + static_cast<int>(gridDim.x) >= units && threadIdx.x == 32) shk::pdl_trigger();
    const Unit w = unit_of(p, u, ntiles);
    // Query rows of this unit -> smem (compute warps only; sQ is free once
    // every compute warp has copied its fragments of the previous unit).
    asm volatile("bar.sync 1, 128;" ::: "memory");
    for (int c = threadIdx.x - 32; c < ROWS * (D / 8); c += 128) {
      const int r = c / (D / 8), cc = c % (D / 8);
      const bool ok = r < w.rows_valid;
      const int rr = ok ? w.row0 + r : w.row0;
      const int tok = rr / G, head = w.h * G + rr % G;
      cp_async16(sQ + swz(r, cc), p.q + (w.qs + tok) * p.q_stride + static_cast<int64_t>(head) * D + cc * 8, ok);
    }
    asm volatile("cp.async.commit_group;\n" ::);
    asm volatile("cp.async.wait_group 0;\n" ::);
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const bool active = rbk * 16 < w.rows_valid;
    uint32_t qf[KSTEPS][4];
    if (active) {
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk)
        ldsm_x4(saddr(sQ) + swz(rbk * 16 + (lane & 15), 2 * kk + (lane >> 4)), qf[kk][0], qf[kk][1], qf[kk][2],
                qf[kk][3]);
    }
    const int ra = rbk * 16 + g, rb = ra + 8;
    const int64_t pa = ra < w.rows_valid ? w.ctx0 + (w.row0 + ra) / G : -1;
    const int64_t pb = rb < w.rows_valid ? w.ctx0 + (w.row0 + rb) / G : -1;
    float o[DT][4];
#pragma unroll
    for (int i = 0; i < DT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    bool bad = false;
    for (int j = w.pg0; j < w.pg1 && !*abort_flag; ++j, ++it) {
      const int st = it % STAGES;
      if (!mbar_wait(&full[st], (it / STAGES) & 1, abort_flag)) {
        if (p.err && lane == 0) atomicCAS(p.err, 0, 12);
        *abort_flag = 1;
        bad = true;
        break;
      }
      const uint32_t kb = saddr(sKV + st * 2 * TILE_BYTES);
      const uint32_t vb = kb + TILE_BYTES;
      if (active) {
        float sc[NT][4];
#pragma unroll
        for (int i = 0; i < NT; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
          for (int np = 0; np < NT / 2; ++np) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4(kb + swz(key0 + np * 16 + (lane & 7) + ((lane >> 4) << 3), 2 * kk + ((lane >> 3) & 1)), b0, b1,
                    b2, b3);
            mma16816(sc[2 * np], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
            mma16816(sc[2 * np + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
          }
        }
        const int64_t kbase = static_cast<int64_t>(j) * KEYS + key0;
        const bool edge = kbase + KEYS / KS - 1 > min(pa, pb) || pa < 0 || pb < 0;
        float mx_a = m_a, mx_b = m_b;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int64_t kp = kbase + nt * 8 + 2 * t4 + e;
            float va = sc[nt][e] * p.scale_log2, vb2 = sc[nt][2 + e] * p.scale_log2;
            if (edge) {
              if (kp > pa) va = -INFINITY;
              if (kp > pb) vb2 = -INFINITY;
            }
            sc[nt][e] = va;
            sc[nt][2 + e] = vb2;
            mx_a = fmaxf(mx_a, va);
            mx_b = fmaxf(mx_b, vb2);
          }
        }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        const float base_a = mx_a == -INFINITY ? 0.f : mx_a;
        const float base_b = mx_b == -INFINITY ? 0.f : mx_b;
        const float al_a = exp2f(m_a - base_a), al_b = exp2f(m_b - base_b);
        m_a = mx_a;
        m_b = mx_b;
        float sum_a = 0.f, sum_b = 0.f;
        uint32_t pf[KC][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float p0 = exp2f(sc[nt][0] - base_a), p1 = exp2f(sc[nt][1] - base_a);
          const float p2 = exp2f(sc[nt][2] - base_b), p3 = exp2f(sc[nt][3] - base_b);
          sum_a += p0 + p1;
          sum_b += p2 + p3;
          pf[nt >> 1][(nt & 1) * 2 + 0] = pack2(p0, p1);
          pf[nt >> 1][(nt & 1) * 2 + 1] = pack2(p2, p3);
        }
        l_a = l_a * al_a + sum_a;
        l_b = l_b * al_b + sum_b;
#pragma unroll
        for (int dt = 0; dt < DT; ++dt) {
          o[dt][0] *= al_a;
          o[dt][1] *= al_a;
          o[dt][2] *= al_b;
          o[dt][3] *= al_b;
        }
#pragma unroll
        for (int kc = 0; kc < KC; ++kc) {
#pragma unroll
          for (int dp = 0; dp < DT / 2; ++dp) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vb + swz(key0 + kc * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), 2 * dp + (lane >> 4)), b0,
                      b1, b2, b3);
            mma16816(o[2 * dp], pf[kc][0], pf[kc][1], pf[kc][2], pf[kc][3], b0, b1);
            mma16816(o[2 * dp + 1], pf[kc][0], pf[kc][1], pf[kc][2], pf[kc][3], b2, b3);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    (void)bad;  // an aborted unit still takes part in every named barrier below; its stores are skipped
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
    if (KS > 1) {
      float* xs = sMerge + (cw * 32 + lane) * (DT * 4 + 4);
      if (kpart != 0 && active) {
#pragma unroll
        for (int dt = 0; dt < DT; ++dt)
#pragma unroll
          for (int e = 0; e < 4; ++e) xs[dt * 4 + e] = o[dt][e];
        xs[DT * 4 + 0] = m_a;
        xs[DT * 4 + 1] = m_b;
        xs[DT * 4 + 2] = l_a;
        xs[DT * 4 + 3] = l_b;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (kpart == 0 && active) {
#pragma unroll
        for (int q = 1; q < KS; ++q) {
          const float* ys = sMerge + ((cw + q) * 32 + lane) * (DT * 4 + 4);
          const float mq_a = ys[DT * 4 + 0], mq_b = ys[DT * 4 + 1];
          const float na = fmaxf(m_a, mq_a), nb = fmaxf(m_b, mq_b);
          const float ba = na == -INFINITY ? 0.f : na, bb = nb == -INFINITY ? 0.f : nb;
          const float sa = exp2f(m_a - ba), sb = exp2f(m_b - bb);
          const float qa = exp2f(mq_a - ba), qb = exp2f(mq_b - bb);
#pragma unroll
          for (int dt = 0; dt < DT; ++dt) {
            o[dt][0] = o[dt][0] * sa + ys[dt * 4 + 0] * qa;
            o[dt][1] = o[dt][1] * sa + ys[dt * 4 + 1] * qa;
            o[dt][2] = o[dt][2] * sb + ys[dt * 4 + 2] * qb;
            o[dt][3] = o[dt][3] * sb + ys[dt * 4 + 3] * qb;
          }
          l_a = l_a * sa + ys[DT * 4 + 2] * qa;
          l_b = l_b * sb + ys[DT * 4 + 3] * qb;
          m_a = na;
          m_b = nb;
        }
      }
    }
    if (kpart != 0 || !active || *abort_flag) continue;
    const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f;
    const float inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = half ? rb : ra;
      if (r >= w.rows_valid) continue;
      const int rr = w.row0 + r;
      const int64_t tok = w.qs + rr / G;
      const int head = w.h * G + rr % G;
      const float inv = half ? inv_b : inv_a;
      if (p.nsplit == 1) {
        __nv_bfloat16* dst = p.out + tok * p.out_stride + static_cast<int64_t>(head) * D;
#pragma unroll
        for (int dt = 0; dt < DT; ++dt)
          *reinterpret_cast<__nv_bfloat162*>(dst + dt * 8 + 2 * t4) =
              __floats2bfloat162_rn(o[dt][2 * half] * inv, o[dt][2 * half + 1] * inv);
      } else {
        // Partial: normalised O and (max, sum) in log2 units, per (row, split).
        const int64_t prow = (tok * p.hq + head) * p.nsplit + w.split;
        float* dst = p.part_o + prow * D;
#pragma unroll
        for (int dt = 0; dt < DT; ++dt)
          *reinterpret_cast<float2*>(dst + dt * 8 + 2 * t4) =
              make_float2(o[dt][2 * half] * inv, o[dt][2 * half + 1] * inv);
        if (t4 == 0) {
          p.part_ml[prow * 2] = half ? m_b : m_a;
          p.part_ml[prow * 2 + 1] = half ? l_b : l_a;
        }
      }
    }
  }
}

// One warp per (token, q head): combine nsplit partials in split order.
template <int D>
__global__ void attn_merge_kernel(__nv_bfloat16* __restrict__ out, int64_t out_stride, const float* __restrict__ part_o,
                                  const float* __restrict__ part_ml, int64_t rows, int hq, int nsplit) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  const float* ml = part_ml + w * nsplit * 2;
  float mx = -INFINITY;
  for (int s = 0; s < nsplit; ++s)
    if (ml[2 * s + 1] > 0.f) mx = fmaxf(mx, ml[2 * s]);
  float acc[D / 32];
#pragma unroll
  for (int i = 0; i < D / 32; ++i) acc[i] = 0.f;
  float den = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float l = ml[2 * s + 1];
    if (!(l > 0.f)) continue;
    const float wgt = exp2f(ml[2 * s] - mx) * l;
    den += wgt;
    const float* po = part_o + (w * nsplit + s) * D;
#pragma unroll
    for (int i = 0; i < D / 32; ++i) acc[i] += wgt * po[lane + 32 * i];
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  const int64_t tok = w / hq;
  const int head = static_cast<int>(w % hq);
  __nv_bfloat16* dst = out + tok * out_stride + static_cast<int64_t>(head) * D;
#pragma unroll
  for (int i = 0; i < D / 32; ++i) dst[lane + 32 * i] = __float2bfloat16(acc[i] * inv);
}

}  // namespace attn
}  // namespace shk

using namespace shk::attn;

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

// Cache viewed as rows of D bf16: dims {D, rows}, box {64, 64}, 128-byte swizzle.
int cache_map(CUtensorMap* m, const void* base, int64_t rows, int d) {
  auto enc = encoder();
  if (!enc) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(d) * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

template <int D, int KS>
int launch_ks(const CUtensorMap& mk, const CUtensorMap& mv, const AttnParams& p, int ntiles, cudaStream_t st) {
  constexpr int STAGES = Stages<D, KS>::value;
  constexpr int MERGE = KS > 1 ? 4 * 32 * (D / 8 * 4 + 4) * 4 : 0;
  constexpr int SMEM = 1024 + 64 * D * 2 * (1 + 2 * STAGES) + MERGE + 2 * STAGES * 8 + 16;
  static_assert(SMEM <= 227 * 1024, "paged attention shared-memory budget exceeds 227 KB per block");
  const int smem = SMEM;
  auto k = paged_attn_kernel<D, KS>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return 300 + static_cast<int>(e);
  static int num_sms = 0;
  if (!num_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int units = ntiles * p.hk * p.nsplit;
  const int grid = units < num_sms ? units : num_sms;
  shk::launch(k, dim3(grid), dim3(THREADS), smem, st, mk, mv, p, ntiles);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : 400 + static_cast<int>(e);
}

template <int D>
int launch(const AttnParams& p, int ntiles, int cache_rows, int max_rows, cudaStream_t st) {
  CUtensorMap mk, mv;
  int r = cache_map(&mk, p.k_cache, cache_rows, D);
  if (r) return 100 + r;
  r = cache_map(&mv, p.v_cache, cache_rows, D);
  if (r) return 200 + r;
  if constexpr (D == 256) {
    // The key-split merge area does not fit next to a 256-wide page ring.
    r = launch_ks<D, 1>(mk, mv, p, ntiles, st);
  } else {
    r = max_rows <= 16 ? launch_ks<D, 4>(mk, mv, p, ntiles, st)
                       : (max_rows <= 32 ? launch_ks<D, 2>(mk, mv, p, ntiles, st) : launch_ks<D, 1>(mk, mv, p, ntiles, st));
  }
  if (r) return r;
  cudaError_t e;
  if (p.nsplit > 1) {
    const int64_t rows = p.num_tokens * p.hq;
    const int64_t threads = rows * 32;
    shk::launch(attn_merge_kernel<D>, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0, st, 
        p.out, p.out_stride, p.part_o, p.part_ml, rows, p.hq, p.nsplit);
    e = cudaGetLastError();
    if (e != cudaSuccess) return 500 + static_cast<int>(e);
  }
  return 0;
}
}  // namespace

extern "C" int sh_paged_attention(const AttnParams* params, int ntiles, int num_blocks, int head_dim, int max_rows,
                                  cudaStream_t stream) {
  const AttnParams& p = *params;
  if (ntiles <= 0 || p.num_tokens <= 0) return 0;
  if (p.nsplit < 1 || p.hq % p.hk != 0) return -1;
  if (p.nsplit > 1 && (p.part_o == nullptr || p.part_ml == nullptr)) return -2;
  if ((reinterpret_cast<uintptr_t>(p.k_cache) & 15) || (reinterpret_cast<uintptr_t>(p.v_cache) & 15)) return -3;
  const int cache_rows = num_blocks * p.hk * KEYS;
  switch (head_dim) {
    case 64:
      return launch<64>(p, ntiles, cache_rows, max_rows, stream);
    case 128:
      return launch<128>(p, ntiles, cache_rows, max_rows, stream);
    case 256:
      return launch<256>(p, ntiles, cache_rows, max_rows, stream);
    default:
      return -4;
  }
}

// ---------------------------------------------------------------------------
// Allocation-free entry point (no counterpart in the reference).
//
// Some callers cannot allocate device memory at the point where they run
// attention: a host runtime without a device allocator of its own (a C or
// Rust serving loop that links only this library), code with a fixed,
// pre-reserved memory budget where a new allocation would fail, or a latency
// path that must not pay cudaMalloc's implicit device synchronisation.  For
// them this variant keeps the split-KV partials in a file-scope device array
// of a fixed size instead of a caller-provided workspace.  The caller still
// passes every input and output buffer.
//
// The array exists once per GPU that loads this library and stays allocated
// until the process exits.  Its device address is looked up with
// cudaGetSymbolAddress on the first call made on each device (with that
// device current); make that first call before any CUDA-graph stream
// capture.  The address is cached together with the device's current
// context: after a cudaDeviceReset the module is loaded again in a new
// context, the change is seen and the address is looked up again (that
// lookup is again a first call: keep it outside a capture).  Every call reuses the same array: calls that overlap on the GPU
// (two streams, two threads) race on it and must be serialised by the
// caller.  Nothing in it needs to start at zero -- every partial slot the
// merge reads is written earlier in the same call.
// ---------------------------------------------------------------------------
namespace {
constexpr int64_t kNoAllocFloats = SH_ATTN_NOALLOC_MAX_FLOATS;
__device__ __align__(256) float g_noalloc_scratch[kNoAllocFloats];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {};
CUcontext g_noalloc_ctx[kMaxDevices] = {};

// cuCtxGetCurrent through the runtime's driver entry point (the library does
// not link libcuda directly, so it loads on machines without a driver).
CUresult current_context(CUcontext* ctx) {
  using Fn = CUresult (*)(CUcontext*);
  static Fn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || p == nullptr)
      return CUDA_ERROR_NOT_FOUND;
    fn = reinterpret_cast<Fn>(p);
  }
  return fn(ctx);
}

int noalloc_scratch(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SH_NOALLOC_ERR_DEVICE;
  // The context may not exist yet before the first lookup (the runtime
  // creates it lazily), so it is read again after cudaGetSymbolAddress.
  CUcontext ctx = nullptr;
  (void)current_context(&ctx);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr || ctx == nullptr || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return SH_NOALLOC_ERR_SYMBOL;
    if (current_context(&ctx) != CUDA_SUCCESS || ctx == nullptr) return SH_NOALLOC_ERR_SYMBOL;
    g_noalloc_ptr[dev] = static_cast<float*>(p);
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}
}  // namespace

extern "C" __attribute__((visibility("default"))) int64_t sh_paged_attention_noalloc_capacity(void) {
  return kNoAllocFloats;
}

extern "C" __attribute__((visibility("default"))) int sh_paged_attention_noalloc(const AttnParams* params, int ntiles,
                                                                                   int num_blocks, int head_dim,
                                                                                   int max_rows, cudaStream_t stream) {
  if (params == nullptr) return SH_NOALLOC_ERR_ARGS;
  AttnParams p = *params;
  if (p.nsplit < 1 || head_dim <= 0 || p.hq <= 0 || p.num_tokens < 0) return SH_NOALLOC_ERR_ARGS;
  p.part_o = nullptr;
  p.part_ml = nullptr;
  if (p.nsplit > 1) {
    // Partials: [rows * nsplit, head_dim] then [rows * nsplit, 2] floats.  The
    // bound is checked by division first, so no product below can overflow.
    const int64_t per_token = static_cast<int64_t>(p.hq) * p.nsplit * (head_dim + 2);
    if (static_cast<int64_t>(p.num_tokens) > kNoAllocFloats / per_token) return SH_NOALLOC_ERR_TOO_LARGE;
    const int64_t slots = static_cast<int64_t>(p.num_tokens) * p.hq * p.nsplit;
    float* base = nullptr;
    const int r = noalloc_scratch(&base);
    if (r) return r;
    p.part_o = base;
    p.part_ml = base + slots * head_dim;
  }
  return sh_paged_attention(&p, ntiles, num_blocks, head_dim, max_rows, stream);
}
