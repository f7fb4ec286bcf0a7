// DeepSeek-V3.2 lightning indexer (DSA) for sm_100a.
//
//   logits[t, p] = ks[p] * sum_h relu(q8[t, h] . k8[p]) * wq[t, h]      (p <= pos_t)
//   topk[t]      = the K largest logits of row t, positions in ascending order
//
// Index keys live in a paged fp8 cache: a 64-key page holds 64 x 128 e4m3 key
// bytes followed by the 64 f32 key scales (8448 bytes, 132 B per key), the
// layout the reference's indexer reads (reference: kernels-oxide/dsa_indexer/
// src/main.rs:1-43, fp8 keys + per-key f32 scale in 64-token pages).
//
// Scoring (dsa_score_kernel) is a persistent tcgen05 kernel, one CTA per SM.
// Work is the flattened list of (row group, 128-key tile) pairs, where a row
// group is up to 384 / IH consecutive query tokens of one request (all MTP /
// verify rows of a decode step), so every key tile is read from HBM once for
// all of those rows.  Each CTA takes an equal contiguous share of the list.
//   warp 0      TMA producer: the row group's fp8 queries and head weights into
//               one of two query buffers, the key tiles (two pages each) into a
//               5-stage ring and their per-key scales into a ring of 8 scale
//               slots, on the same barrier (L2 evict-first: keys are streamed
//               once);
//   warp 1      MMA issuer: D[key, token x head] = K_tile (M = 128 keys) x
//               Q_group^T (N = tokens x IH <= 256) with tcgen05.mma kind::f8f6f4
//               (e4m3 x e4m3 -> f32) into one of two TMEM accumulators, so the
//               epilogue of one group overlaps the MMAs of the next;
//   warps 2..9  two epilogue warpgroups, one per accumulator: each thread owns
//               one key (a TMEM lane) and reduces relu(D) * wq over the heads
//               of each token in registers -- no cross-lane reduction -- then
//               writes the logit with an L2 evict-last hint (the scratch rows,
//               a few tens of MB at decode sizes, stay in L2 for the select).
// Selection (dsa_topk_kernel): one CTA per query token; the row is read once
// from L2 into shared memory, a radix select over 11-bit digits that starts
// below the bits common to the whole row finds the K-th largest logit, and
// one ordered compaction writes the positions.  Equal logits prefer the later
// position.
//
// Every wait is bounded (2 s); a timed-out wait records 400 + phase in *err,
// raises the CTA's abort flag so the other roles leave their loops, and the
// CTA drains its copies in flight and frees its TMEM before it returns.  No TMA
// load here uses cluster multicast.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "dsa_indexer.h"
#include "pdl.cuh"
#include "tcgen05_common.cuh"

namespace shk {
namespace dsa {

using namespace shk::tc;

constexpr int kPage = SH_DSA_PAGE_KEYS;
constexpr int kDim = SH_DSA_DIM;
constexpr int kPageBytes = SH_DSA_PAGE_BYTES;
constexpr int kPageKeyBytes = kPage * kDim;  // 8192
constexpr int kTile = 128;                    // keys per MMA tile (two pages)
constexpr int kTileBytes = kTile * kDim;      // 16 KB
constexpr int kQRows = 384;                   // query rows (token x head) per row group
constexpr int kQBoxRows = 128;                // rows per query TMA box
constexpr int kStages = 5;
constexpr int kThreads = 320;                 // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kAccCols = 256;                 // TMEM columns per accumulator (two accumulators)
// Key scales ride with the key tiles (same full barrier) into a ring of their own.  Slot reuse needs no
// barrier: the producer loads tile g only after the MMA finished tile g - kStages, whose first item waited
// for the epilogue to release the item two items earlier (two accumulators, at most two items per tile),
// so every item of tile g - kStages - 1 had been released; the epilogue reads an item's scales before it
// releases the item, and kScaleSlots > kStages + 1.
constexpr int kScaleSlots = 8;

struct Smem {
  static constexpr int RING = 0;
  static constexpr int QBUF = RING + kStages * kTileBytes;
  static constexpr int QBYTES = kQRows * kDim;
  static constexpr int WQ = QBUF + 2 * QBYTES;
  static constexpr int SCALE = WQ + 2 * kQRows * 4;  // [kScaleSlots][128] key scales, one slot per tile
  static constexpr int BAR = SCALE + kScaleSlots * kTile * 4;
  static constexpr int NBAR = 2 * kStages + 8;
  static constexpr int MISC = BAR + NBAR * 8;
  static constexpr int TOTAL = MISC + 64 + 1024;  // + alignment slack
};
static_assert(Smem::TOTAL <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
// Plain (untiled) bulk copy global -> this CTA's shared memory; sizes and both addresses 16-byte aligned.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// Instruction descriptor for kind::f8f6f4: D f32, A and B e4m3 (format 0), both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_e4m3(int m, int n) {
  return (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}
__device__ __forceinline__ void mma_e4m3(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// tcgen05.wait::ld naming the 32 registers of the outstanding load, so their uses stay after it.
__device__ __forceinline__ void tmem_wait_ld32(float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}
__device__ __forceinline__ void st_evict_last(float* ptr, float v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.f32 [%0], %1, %2;" ::"l"(ptr), "f"(v), "l"(pol) : "memory");
}

// sum_i relu(v[i]) * w[i] over 32 values (w 16-byte aligned shared memory, read as broadcasts).
__device__ __forceinline__ float relu_dot32(const float* v, const float* w) {
  float a = 0.f, b = 0.f;
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const float4 w0 = *reinterpret_cast<const float4*>(w + i);
    const float4 w1 = *reinterpret_cast<const float4*>(w + i + 4);
    a = fmaf(fmaxf(v[i], 0.f), w0.x, a);
    b = fmaf(fmaxf(v[i + 1], 0.f), w0.y, b);
    a = fmaf(fmaxf(v[i + 2], 0.f), w0.z, a);
    b = fmaf(fmaxf(v[i + 3], 0.f), w0.w, b);
    a = fmaf(fmaxf(v[i + 4], 0.f), w1.x, a);
    b = fmaf(fmaxf(v[i + 5], 0.f), w1.y, b);
    a = fmaf(fmaxf(v[i + 6], 0.f), w1.z, a);
    b = fmaf(fmaxf(v[i + 7], 0.f), w1.w, b);
  }
  return a + b;
}

// One (row group, contiguous tile range) piece of a CTA's share of the work.
struct Seg {
  int b;           // request
  int t0, nt;      // first query row, rows in the group
  int64_t pos0;    // position of row t0 (row t0 + j sees keys [0, pos0 + j])
  int64_t last;    // position of the group's last row: keys [0, last] are scored
  int tb, te;      // key tiles [tb, te) of the group
};

// Walks a CTA's share of the flattened (row group, tile) list in order.  Every
// role keeps its own copy; all copies produce the same sequence.
template <int IH>
struct Walk {
  static constexpr int RGT = kQRows / IH;  // query rows per row group
  int b, r, i;
  int64_t left;

  __device__ static int tiles_of(int64_t seq, int64_t ql, int r, int& nt, int64_t& last) {
    const int64_t rest = ql - static_cast<int64_t>(r) * RGT;
    nt = static_cast<int>(rest < RGT ? rest : RGT);
    last = seq - ql + static_cast<int64_t>(r) * RGT + nt - 1;
    return last >= 0 ? static_cast<int>((last + kTile) / kTile) : 0;
  }
  __device__ bool next(Seg& s, const DsaIndexParams& p) {
    while (left > 0 && b < p.B) {
      const int64_t qs = p.q_start[b], ql = p.q_start[b + 1] - qs;
      const int64_t rgn = (ql + RGT - 1) / RGT;
      if (r >= rgn) {
        ++b;
        r = 0;
        i = 0;
        continue;
      }
      int nt;
      int64_t last;
      const int tiles = tiles_of(p.seq_lens[b], ql, r, nt, last);
      if (i >= tiles) {
        ++r;
        i = 0;
        continue;
      }
      const int n = static_cast<int>(tiles - i < left ? tiles - i : left);
      s.b = b;
      s.t0 = static_cast<int>(qs) + r * RGT;
      s.nt = nt;
      s.last = last;
      s.pos0 = last - (nt - 1);
      s.tb = i;
      s.te = i + n;
      i += n;
      left -= n;
      return true;
    }
    return false;
  }
};

// Tiles of request b summed over its row groups.
template <int IH>
__device__ int64_t request_tiles(const DsaIndexParams& p, int b) {
  const int64_t qs = p.q_start[b], ql = p.q_start[b + 1] - qs, seq = p.seq_lens[b];
  int64_t tot = 0;
  const int64_t rgn = (ql + Walk<IH>::RGT - 1) / Walk<IH>::RGT;
  for (int r = 0; r < rgn; ++r) {
    int nt;
    int64_t last;
    tot += Walk<IH>::tiles_of(seq, ql, r, nt, last);
  }
  return tot;
}

template <int IH>
__global__ void __launch_bounds__(kThreads, 1)
    dsa_score_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmS, DsaIndexParams p) {
  static_assert(IH == 16 || IH == 64, "indexer heads");
  constexpr int TPG = kAccCols / IH;  // tokens per MMA group (N <= 256)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Smem::BAR);
  uint64_t* empty = full + kStages;
  uint64_t* accf = empty + kStages;
  uint64_t* acce = accf + 2;
  uint64_t* qfull = acce + 2;
  uint64_t* qfree = qfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Smem::MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int64_t* start = reinterpret_cast<int64_t*>(smem + Smem::MISC + 16);  // b, r, i, count
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 4);   // the four warps of the accumulator's epilogue warpgroup
      mbar_init(&qfull[a], 1);
      mbar_init(&qfree[a], 9);  // MMA commit + the eight epilogue warps
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmK)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmQ)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmS)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(2 * kAccCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // Dependents may launch now: the select kernel waits for this grid's completion anyway.
  shk::pdl_trigger();
  shk::pdl_wait();  // queries, weights and this step's keys come from the preceding kernels
  if (warp == 0) {  // this CTA's share of the flattened (row group, tile) list
    int64_t tot = 0;
    for (int b0 = 0; b0 < p.B; b0 += 32) {
      int64_t v = b0 + lane < p.B ? request_tiles<IH>(p, b0 + lane) : 0;
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      tot += v;
    }
    const int64_t lo = tot * blockIdx.x / gridDim.x, hi = tot * (blockIdx.x + 1) / gridDim.x;
    int64_t acc = 0;
    int sb = p.B;
    int64_t rem = 0;
    for (int b0 = 0; b0 < p.B && sb == p.B; b0 += 32) {
      const int64_t v = b0 + lane < p.B ? request_tiles<IH>(p, b0 + lane) : 0;
      int64_t inc = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t u = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += u;
      }
      const bool mine = v > 0 && acc + inc - v <= lo && lo < acc + inc;
      const unsigned who = __ballot_sync(0xffffffffu, mine);
      if (who) {
        const int src = __ffs(who) - 1;
        sb = b0 + src;
        rem = lo - (acc + __shfl_sync(0xffffffffu, inc - v, src));
      }
      acc += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) {
      int r = 0;
      if (sb < p.B) {
        const int64_t qs = p.q_start[sb], ql = p.q_start[sb + 1] - qs, seq = p.seq_lens[sb];
        for (;; ++r) {
          int nt;
          int64_t last;
          const int tl = Walk<IH>::tiles_of(seq, ql, r, nt, last);
          if (rem < tl) break;
          rem -= tl;
        }
      }
      start[0] = sb;
      start[1] = r;
      start[2] = rem;
      start[3] = sb < p.B ? hi - lo : 0;
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;
  Walk<IH> walk{static_cast<int>(start[0]), static_cast<int>(start[1]), static_cast<int>(start[2]), start[3]};
  auto raise = [&](int code) {
    if (p.err) atomicCAS(p.err, 0, code);
    *abort_flag = 1;
  };
  uint8_t* ring = smem + Smem::RING;
  uint8_t* qbuf = smem + Smem::QBUF;
  float* wqbuf = reinterpret_cast<float*>(smem + Smem::WQ);
  float* sscale = reinterpret_cast<float*>(smem + Smem::SCALE);

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_k = policy_evict_first(), pol_q = policy_evict_last();
      int stage = 0, phase = 0, si = 0;
      uint32_t g = 0;  // tiles loaded by this CTA (scale slot g % kScaleSlots)
      Seg s;
      bool ok = true;
      while (ok && walk.next(s, p)) {
        const int qb = si & 1;
        if (si >= 2 && !mbar_wait(&qfree[qb], ((si >> 1) - 1) & 1, abort_flag)) {
          raise(402);
          break;
        }
        const int rows = s.nt * IH, boxes = (rows + kQBoxRows - 1) / kQBoxRows;
        mbar_expect_tx(&qfull[qb], boxes * kQBoxRows * kDim + rows * 4);
        for (int c = 0; c < boxes; ++c)
          tma_load_2d_hint(qbuf + qb * Smem::QBYTES + c * kQBoxRows * kDim, &tmQ, 0, s.t0 * IH + c * kQBoxRows,
                           &qfull[qb], pol_q);
        bulk_load(wqbuf + qb * kQRows, p.wq + static_cast<int64_t>(s.t0) * IH, rows * 4, &qfull[qb]);
        const int32_t* bt = p.block_tables + static_cast<int64_t>(s.b) * p.bt_stride;
        for (int tile = s.tb; tile < s.te; ++tile) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            raise(401);
            ok = false;
            break;
          }
          const int pg = 2 * tile;
          const bool two = static_cast<int64_t>(pg + 1) * kPage <= s.last;
          mbar_expect_tx(&full[stage], (two ? 2 : 1) * (kPageKeyBytes + kPage * 4));
          uint8_t* dst = ring + stage * kTileBytes;
          float* sdst = sscale + (g % kScaleSlots) * kTile;
          tma_load_3d_hint(dst, &tmK, 0, 0, bt[pg], &full[stage], pol_k);
          tma_load_2d_hint(sdst, &tmS, 0, bt[pg], &full[stage], pol_k);
          if (two) {
            tma_load_3d_hint(dst + kPageKeyBytes, &tmK, 0, 0, bt[pg + 1], &full[stage], pol_k);
            tma_load_2d_hint(sdst + kPage, &tmS, 0, bt[pg + 1], &full[stage], pol_k);
          }
          ++g;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        ++si;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0, phase = 0, si = 0;
      uint32_t j = 0;  // accumulator use counter (buffer j & 1)
      Seg s;
      bool ok = true;
      while (ok && walk.next(s, p)) {
        const int qb = si & 1;
        if (!mbar_wait(&qfull[qb], (si >> 1) & 1, abort_flag)) {
          raise(403);
          break;
        }
        fence_after();
        const int ng = (s.nt + TPG - 1) / TPG, tpg = (s.nt + ng - 1) / ng;
        const uint32_t qaddr = smem_addr(qbuf + qb * Smem::QBYTES);
        for (int tile = s.tb; tile < s.te && ok; ++tile) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            raise(404);
            ok = false;
            break;
          }
          fence_after();
          const uint32_t kaddr = smem_addr(ring + stage * kTileBytes);
          for (int g = 0; g < ng; ++g, ++j) {
            const uint32_t buf = j & 1, use = j >> 1;
            if (use >= 1 && !mbar_wait(&acce[buf], (use - 1) & 1, abort_flag)) {
              raise(405);
              ok = false;
              break;
            }
            fence_after();
            const int n = min(tpg, s.nt - g * tpg) * IH;
            const uint32_t idesc = idesc_e4m3(kTile, n);
            // descriptors built once and advanced by (32 bytes / 16) per k-step
            const uint64_t adesc = sw128_desc(kaddr), bdesc = sw128_desc(qaddr + g * tpg * IH * kDim);
#pragma unroll
            for (int k = 0; k < kDim / 32; ++k)
              mma_e4m3(tmem_base + buf * kAccCols, adesc + static_cast<uint64_t>(2 * k), bdesc + static_cast<uint64_t>(2 * k),
                       idesc, k > 0 ? 1u : 0u);
            mma_commit(&accf[buf]);
          }
          if (!ok) break;
          mma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        mma_commit(&qfree[qb]);
        ++si;
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue warpgroups
    const int e = (warp - 2) >> 2;       // accumulator / warpgroup
    const int qtr = warp & 3;            // TMEM lane quarter this warp may access
    const int row = qtr * 32 + lane;     // key within the tile
    const uint64_t pol_l = policy_evict_last();
    int si = 0;
    uint32_t j = 0;
    uint32_t gt = 0;  // tiles of this CTA before the current one (scale slot gt % kScaleSlots)
    Seg s;
    bool ok = true;
    while (ok && walk.next(s, p)) {
      const int qb = si & 1;
      const int ng = (s.nt + TPG - 1) / TPG, tpg = (s.nt + ng - 1) / ng;
      const float* wq = wqbuf + qb * kQRows;
      for (int tile = s.tb; tile < s.te && ok; ++tile, ++gt) {
        const int64_t pos = static_cast<int64_t>(tile) * kTile + row;
        for (int g = 0; g < ng; ++g, ++j) {
          if ((j & 1) != static_cast<uint32_t>(e)) continue;
          const uint32_t use = j >> 1;
          // the warp agrees on the outcome: the TMEM loads below (.sync.aligned) run on all lanes or none
          if (!__all_sync(0xffffffffu, mbar_wait(&accf[e], use & 1, abort_flag))) {
            raise(406);
            ok = false;
            break;
          }
          fence_after();
          // this key's scale (pages past the group's last key were not loaded: their keys are never stored)
          const float ks = sscale[(gt % kScaleSlots) * kTile + row];
          const int ntok = min(tpg, s.nt - g * tpg);
          const uint32_t tb = tmem_base + (static_cast<uint32_t>(qtr * 32) << 16) + e * kAccCols;
          const float* w = wq + g * tpg * IH;
          const int jt0 = g * tpg;  // first row of the group within the row group
          if constexpr (IH == 64) {
            float va[32], vb[32];
            tmem_ld32_nowait(tb, va);
            tmem_wait_ld32(va);
            for (int tok = 0; tok < ntok; ++tok) {
              tmem_ld32_nowait(tb + tok * 64 + 32, vb);
              float acc = relu_dot32(va, w + tok * 64);
              tmem_wait_ld32(vb);
              if (tok + 1 < ntok) tmem_ld32_nowait(tb + (tok + 1) * 64, va);
              acc += relu_dot32(vb, w + tok * 64 + 32);
              const int64_t lim = s.pos0 + jt0 + tok;
              if (pos <= lim) st_evict_last(p.logits + (s.t0 + jt0 + tok) * p.ld + pos, acc * ks, pol_l);
              if (tok + 1 < ntok) tmem_wait_ld32(va);
            }
          } else {
            float va[32];
            for (int c = 0; c < ntok; c += 2) {  // 32 columns = two tokens of 16 heads
              tmem_ld32_nowait(tb + c * 16, va);
              tmem_wait_ld32(va);
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int tok = c + h;
                if (tok < ntok) {
                  float acc = 0.f;
#pragma unroll
                  for (int i = 0; i < 16; ++i) acc = fmaf(fmaxf(va[h * 16 + i], 0.f), w[tok * 16 + i], acc);
                  const int64_t lim = s.pos0 + jt0 + tok;
                  if (pos <= lim) st_evict_last(p.logits + (s.t0 + jt0 + tok) * p.ld + pos, acc * ks, pol_l);
                }
              }
            }
          }
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce[e]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&qfree[qb]);  // this warp no longer reads the group's weights
      ++si;
    }
  }
  if (warp == 0 && lane == 0 && *abort_flag) {
    // Loads issued before the abort complete within microseconds; give them 200 us.
    const uint64_t t0 = now_ns();
    while (now_ns() - t0 < 200000) {
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(2 * kAccCols));
  }
}

// ------------------------------------------------------------------------------ top-k select
constexpr int kSelThreads = 1024;
constexpr int kBins = 2048;
constexpr int kSelMaxStaged = 40960;  // rows of up to this many keys are staged in shared memory (160 KB)

__device__ __forceinline__ uint32_t ordered_bits(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // larger float -> larger unsigned
}

__device__ __forceinline__ int request_of(const int64_t* q_start, int B, int t) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (q_start[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Block-wide exclusive prefix sum of one value per thread; *total gets the sum.
__device__ __forceinline__ int block_excl_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += u;
  }
  if (lane == 31) warp_sums[warp] = inc;
  __syncthreads();
  int before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < kSelThreads / 32; ++w) {
    const int sw = warp_sums[w];
    before += w < warp ? sw : 0;
    all += sw;
  }
  __syncthreads();  // warp_sums may be reused
  *total = all;
  return before + inc - v;
}

// One CTA per query row.  Pass 0 reads the logits row once (float4, L2) into shared memory as orderable
// keys (rows longer than `staged` keys are re-read from global memory instead) and finds the row's
// smallest and largest key.  The radix select then starts at the highest bit in which those two differ
// (the bits above it are common to every key), so the first 11-bit digit already spreads the keys over
// the histogram instead of piling them into a few exponent bins; at most three digit passes follow.  One
// ordered compaction writes the selected positions.
__global__ void __launch_bounds__(kSelThreads) dsa_topk_kernel(DsaIndexParams p, int staged) {
  shk::pdl_trigger();
  shk::pdl_wait();
  extern __shared__ uint4 sel_smem[];
  uint32_t* skeys = reinterpret_cast<uint32_t*>(sel_smem);
  __shared__ uint32_t hist[kBins];
  __shared__ int warp_sums[kSelThreads / 32];
  __shared__ uint32_t red[2][kSelThreads / 32];
  __shared__ uint32_t pick[4];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t = blockIdx.x;
  const int b = request_of(p.q_start, p.B, t);
  const int64_t qs = p.q_start[b], ql = p.q_start[b + 1] - qs, seq = p.seq_lens[b];
  const int64_t n64 = seq - ql + (t - qs) + 1;
  const int n = static_cast<int>(n64 > 0 ? n64 : 0);
  int32_t* out = p.topk + static_cast<int64_t>(t) * p.K;
  if (n <= p.K) {  // every causal key is selected
    for (int i = tid; i < p.K; i += kSelThreads) out[i] = i < n ? i : -1;
    return;
  }
  const float* row = p.logits + static_cast<int64_t>(t) * p.ld;
  const bool in_smem = n <= staged;
  auto key_at = [&](int i) -> uint32_t { return in_smem ? skeys[i] : ordered_bits(__ldcg(row + i)); };

  uint32_t kmin = 0xffffffffu, kmax = 0u;
  for (int i0 = 4 * tid; i0 < n; i0 += 4 * kSelThreads) {
    uint32_t u[4];
    if (i0 + 3 < n) {
      const float4 f = __ldcg(reinterpret_cast<const float4*>(row + i0));
      u[0] = ordered_bits(f.x);
      u[1] = ordered_bits(f.y);
      u[2] = ordered_bits(f.z);
      u[3] = ordered_bits(f.w);
      if (in_smem) *reinterpret_cast<uint4*>(skeys + i0) = make_uint4(u[0], u[1], u[2], u[3]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        u[e] = i0 + e < n ? ordered_bits(__ldcg(row + i0 + e)) : 0u;
        if (in_smem && i0 + e < n) skeys[i0 + e] = u[e];
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (i0 + e < n) {
        kmin = min(kmin, u[e]);
        kmax = max(kmax, u[e]);
      }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
    kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
  }
  if (lane == 0) {
    red[0][warp] = kmin;
    red[1][warp] = kmax;
  }
  __syncthreads();  // also publishes the staged keys
  kmin = 0xffffffffu;
  kmax = 0u;
#pragma unroll
  for (int w = 0; w < kSelThreads / 32; ++w) {
    kmin = min(kmin, red[0][w]);
    kmax = max(kmax, red[1][w]);
  }
  const uint32_t diff = kmin ^ kmax;
  int hb = diff ? 31 - __clz(diff) : -1;  // highest bit not common to every key
  uint32_t mask = hb >= 31 ? 0u : ~((2u << hb) - 1u);
  if (hb < 0) mask = 0xffffffffu;
  uint32_t prefix = kmax & mask, eq_total = static_cast<uint32_t>(n);
  int remaining = p.K;
  while (hb >= 0) {  // 11-bit digits from bit hb down
    const int shift = hb >= 10 ? hb - 10 : 0, nb = 1 << (hb - shift + 1);
    for (int i = tid; i < nb; i += kSelThreads) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += kSelThreads) {
      const uint32_t u = key_at(i);
      if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & (nb - 1)], 1u);
    }
    __syncthreads();
    if (warp == 0) {  // lane l sums bins [nb - (l + 1) * per, nb - l * per) (counts from the top)
      const int per = nb >= 32 ? nb / 32 : 1;
      const int hi = nb - lane * per;
      uint32_t v = 0;
      if (hi > 0)
        for (int d = hi - 1; d >= hi - per; --d) v += hist[d];
      uint32_t inc = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t u = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += u;
      }
      const bool cross = hi > 0 && inc >= static_cast<uint32_t>(remaining) &&
                         inc - v < static_cast<uint32_t>(remaining);
      if (cross) {
        uint32_t above = inc - v;
        int d = hi - 1;
        for (; d > hi - per; --d) {
          if (above + hist[d] >= static_cast<uint32_t>(remaining)) break;
          above += hist[d];
        }
        pick[0] = static_cast<uint32_t>(d);
        pick[1] = static_cast<uint32_t>(remaining) - above;
        pick[2] = hist[d];
      }
    }
    __syncthreads();
    prefix |= pick[0] << shift;
    mask |= static_cast<uint32_t>(nb - 1) << shift;
    remaining = static_cast<int>(pick[1]);
    eq_total = pick[2];
    hb = shift - 1;
    __syncthreads();
  }
  // prefix is the K-th largest key: take every key above it and the `remaining` latest keys equal to it,
  // in ascending position order (chunks of 8 consecutive keys per thread).
  const int skip = static_cast<int>(eq_total) - remaining;
  int base_pos = 0, base_eq = 0;
  for (int c0 = 0; c0 < n; c0 += 8 * kSelThreads) {
    const int i0 = c0 + 8 * tid;
    uint32_t gt = 0, eq = 0;  // bit e: key i0 + e above / equal to the threshold
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t u = i0 + e < n ? key_at(i0 + e) : 0u;
      gt |= static_cast<uint32_t>(i0 + e < n && u > prefix) << e;
      eq |= static_cast<uint32_t>(i0 + e < n && u == prefix) << e;
    }
    int tot_eq, tot_sel;
    const int eq_before = base_eq + block_excl_scan(__popc(eq), warp_sums, &tot_eq);
    uint32_t sel = gt;
    int e_cnt = eq_before;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if ((eq >> e) & 1u) sel |= static_cast<uint32_t>(e_cnt++ >= skip) << e;
    int pos = base_pos + block_excl_scan(__popc(sel), warp_sums, &tot_sel);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if ((sel >> e) & 1u) {
        if (pos < p.K) out[pos] = i0 + e;
        ++pos;
      }
    base_pos += tot_sel;
    base_eq += tot_eq;
  }
  for (int i = base_pos + tid; i < p.K; i += kSelThreads) out[i] = -1;
}

// ------------------------------------------------------------------------------ quantisation
__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  uint32_t out;
  asm("{\n .reg .b16 lo, hi;\n"
      " cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n"
      " cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n"
      " mov.b32 %0, {lo, hi};\n}"
      : "=r"(out)
      : "f"(a), "f"(b), "f"(c), "f"(d));
  return out;
}

// One warp per 128-value row: s = amax / 448 (1 for an all-zero row), bytes = e4m3(x / s), round to
// nearest even with saturation.  Divisions are IEEE (div.rn), so the host reference reproduces the codes.
__device__ __forceinline__ float quant_row(const __nv_bfloat16* src, uint8_t* dst, int lane) {
  const uint2 raw = *reinterpret_cast<const uint2*>(src + lane * 4);
  const __nv_bfloat162 h0 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
  const __nv_bfloat162 h1 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
  const float x0 = __low2float(h0), x1 = __high2float(h0), x2 = __low2float(h1), x3 = __high2float(h1);
  float am = fmaxf(fmaxf(fabsf(x0), fabsf(x1)), fmaxf(fabsf(x2), fabsf(x3)));
#pragma unroll
  for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  const float s = am > 0.f ? __fdiv_rn(am, 448.f) : 1.f;
  *reinterpret_cast<uint32_t*>(dst + lane * 4) =
      e4m3x4(__fdiv_rn(x0, s), __fdiv_rn(x1, s), __fdiv_rn(x2, s), __fdiv_rn(x3, s));
  return s;
}

__global__ void dsa_cache_write_kernel(uint8_t* __restrict__ cache, const __nv_bfloat16* __restrict__ k,
                                       int64_t k_stride, const int64_t* __restrict__ slots, int T) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= T) return;
  const int64_t slot = slots[t];
  if (slot < 0) return;
  uint8_t* page = cache + (slot / kPage) * kPageBytes;
  const int r = static_cast<int>(slot % kPage);
  const float s = quant_row(k + t * k_stride, page + r * kDim, lane);
  if (lane == 0) *reinterpret_cast<float*>(page + kPageKeyBytes + r * 4) = s;
}

__global__ void dsa_quant_q_kernel(uint8_t* __restrict__ q8, float* __restrict__ wq,
                                   const __nv_bfloat16* __restrict__ q, const float* __restrict__ w, int rows) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float s = quant_row(q + static_cast<int64_t>(r) * kDim, q8 + static_cast<int64_t>(r) * kDim, lane);
  if (lane == 0) wq[r] = w[r] * s;
}

}  // namespace dsa
}  // namespace shk

namespace {

using namespace shk::dsa;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

constexpr int kMaxDevices = 64;

template <int IH>
int launch_score(const DsaIndexParams& p, cudaStream_t st) {
  auto enc = encode_fn();
  if (!enc) return -1;
  CUtensorMap mk, mq;
  {  // keys: {128 bytes, 64 keys, pages}, one page per box
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(kDim), static_cast<cuuint64_t>(kPage),
                          static_cast<cuuint64_t>(p.num_pages)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(kDim), static_cast<cuuint64_t>(kPageBytes)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(kDim), static_cast<cuuint32_t>(kPage), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = enc(&mk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(p.kcache), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return 1000 + static_cast<int>(r);
  }
  {  // queries: {128 bytes, T * IH rows}
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(kDim), static_cast<cuuint64_t>(p.T) * IH};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(kDim)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kDim), static_cast<cuuint32_t>(kQBoxRows)};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&mq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(p.q8), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return 2000 + static_cast<int>(r);
  }
  CUtensorMap ms;
  {  // key scales: {64 floats, pages}, starting after each page's key bytes
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(kPage), static_cast<cuuint64_t>(p.num_pages)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(kPageBytes)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kPage), 1};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<uint8_t*>(p.kcache + kPageKeyBytes),
                           dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return 3000 + static_cast<int>(r);
  }
  auto k = dsa_score_kernel<IH>;
  static bool ready[kMaxDevices] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = 0;
  if (!ready[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::TOTAL);
    if (e != cudaSuccess) return static_cast<int>(e);
    ready[dev] = true;
  }
  shk::launch(k, dim3(p.grid), dim3(kThreads), Smem::TOTAL, st, mk, mq, ms, p);
  return static_cast<int>(cudaGetLastError());
}

int check(const DsaIndexParams* p) {
  if (!p->q8 || !p->wq || !p->kcache || !p->logits || !p->block_tables || !p->seq_lens || !p->q_start) return -1;
  if (p->IH != 16 && p->IH != 64) return -2;
  if (p->grid < 1 || p->num_pages < 1 || p->B < 1) return -3;
  if (p->ld % 4 != 0) return -4;
  if ((reinterpret_cast<uintptr_t>(p->kcache) | reinterpret_cast<uintptr_t>(p->q8) |
       reinterpret_cast<uintptr_t>(p->wq)) & 15)
    return -5;
  return 0;
}

}  // namespace

extern "C" int sh_dsa_cache_write(uint8_t* cache, const __nv_bfloat16* k, int64_t k_stride, const int64_t* slots,
                                  int T, cudaStream_t stream) {
  if (T <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(k) & 7) || (k_stride & 3)) return -1;
  shk::launch(dsa_cache_write_kernel, dim3((T + 7) / 8), dim3(256), 0, stream, cache, k, k_stride, slots, T);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_dsa_quant_q(uint8_t* q8, float* wq, const __nv_bfloat16* q, const float* w, int rows,
                              cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (reinterpret_cast<uintptr_t>(q) & 7) return -1;
  shk::launch(dsa_quant_q_kernel, dim3((rows + 7) / 8), dim3(256), 0, stream, q8, wq, q, w, rows);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_dsa_score(const DsaIndexParams* p, cudaStream_t stream) {
  if (p->T <= 0) return 0;
  const int c = check(p);
  if (c) return c;
  return p->IH == 64 ? launch_score<64>(*p, stream) : launch_score<16>(*p, stream);
}

extern "C" int sh_dsa_index(const DsaIndexParams* p, cudaStream_t stream) {
  if (p->T <= 0) return 0;
  if (p->K <= 0 || !p->topk) return -1;
  const int r = sh_dsa_score(p, stream);
  if (r) return r;
  // rows of up to max_keys keys are staged in shared memory (capped at 160 KB)
  const int staged = static_cast<int>(p->ld < kSelMaxStaged ? p->ld : kSelMaxStaged);
  static bool ready[kMaxDevices] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = 0;
  if (!ready[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(dsa_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSelMaxStaged * 4);
    if (e != cudaSuccess) return static_cast<int>(e);
    ready[dev] = true;
  }
  shk::launch(dsa_topk_kernel, dim3(p->T), dim3(kSelThreads), static_cast<size_t>(staged) * 4, stream, *p, staged);
  return static_cast<int>(cudaGetLastError());
}
