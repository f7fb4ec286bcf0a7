// BF16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
//   D[i, j] = sum_k P[i, k] * Q[j, k]      P: [rows_p, K], Q: [rows_q, K] (both K-major)
//
// P feeds the MMA's A side in 128-row tiles, Q the B side in BN-row tiles.
// Normal orientation stores out[i, j]; TRANS stores out[j, i] so the same
// kernel serves y = x W^T with the activations on either side ("swap-AB":
// for small token counts the weights take the 128-row side and the tokens
// become the MMA N dimension).
//
// Structure (one CTA per SM, persistent over work units):
//   warp 0      : TMA producer -- 128B-swizzled [rows][64] bf16 tiles of P and
//                 Q into a STAGES-deep smem ring, completion via mbarrier tx
//                 counts.  No TMA load uses cluster multicast.
//   warp 1      : TMEM allocator and single-thread MMA issuer:
//                 tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) x4
//                 per 64-wide k-block into one of two TMEM accumulators,
//                 tcgen05.commit frees the smem stage / publishes the tile.
//   warps 2..5  : epilogue -- tcgen05.ld 32x32b (each warp owns its 32-lane
//                 TMEM sub-partition), bf16 convert, global store; the second
//                 accumulator lets tile t's epilogue overlap tile t+1's MMAs.
// Split-K (SPLIT=true) writes fp32 partials [splits][rows_p][rows_q] to a
// workspace; gemm_splitk_reduce sums them in a fixed order (deterministic).
// Every mbarrier wait is bounded: on timeout the kernel records an error code
// in *err, stops issuing work, drains and frees TMEM, and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm_tcgen05.h"
#include "tcgen05_common.cuh"
#include "pdl.cuh"

namespace shk {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;

// Instruction descriptor: D f32, A/B bf16, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) { return idesc_bf16_mn(BM, n); }

template <int BN>
__host__ __device__ constexpr int tmem_cols() {
  return (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
}

// Push-epilogue staging: per epilogue warp 32 rows x 64 columns of bf16, rows
// padded to 72 elements (144 B) so the 32 lanes' row writes spread over banks.
constexpr int PUSH_LD = 72;
constexpr int PUSH_STAGE_BYTES = 4 * 32 * PUSH_LD * 2;

template <int BN, int STAGES, bool PUSH = false>
struct Smem {
  static constexpr int P_BYTES = BM * BK * 2;
  static constexpr int Q_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = P_BYTES + Q_BYTES;
  static constexpr int PUSH_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = PUSH_OFF + (PUSH ? PUSH_STAGE_BYTES : 0);
  static constexpr int TOTAL = BAR_OFF + (2 * STAGES + 5) * 8 + 16 + 1024;  // + alignment slack
  static_assert(TOTAL <= 227 * 1024, "shared memory budget");
};

struct Work {
  int tp, tq, sp;
  int p_y, q_y;       // TMA row coordinates of the P and Q tiles
  int p_lim, q_lim;   // valid rows: p < p_lim (tile-local base tp*BM), q in [q_y, q_lim)
  int q_base;         // output row base for q
};

__device__ __forceinline__ Work decode_work(int w, const GemmParams& g, int bn) {
  Work r;
  if (g.groups) {
    const int4 e = g.groups[w / g.tiles_p];
    r.sp = 0;
    r.tp = w % g.tiles_p;
    r.tq = 0;
    r.p_y = e.z + r.tp * BM;
    r.q_y = e.x;
    r.p_lim = g.rows_p;
    r.q_lim = e.x + e.y;
    r.q_base = e.x;
    return r;
  }
  const int tiles = g.tiles_p * g.tiles_q;
  r.sp = w / tiles;
  const int t = w % tiles;
  if (g.p_fast) {
    r.tp = t % g.tiles_p;
    r.tq = t / g.tiles_p;
  } else {
    r.tq = t % g.tiles_q;
    r.tp = t / g.tiles_q;
  }
  r.p_y = r.tp * BM;
  r.q_y = r.tq * bn;
  r.p_lim = g.rows_p;
  r.q_lim = g.rows_q;
  r.q_base = r.tq * bn;
  return r;
}

template <int BN, int STAGES, bool TRANS, bool SPLIT, bool PUSH = false>
__global__ void __launch_bounds__(192, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmQ, GemmParams g) {
  using S = Smem<BN, STAGES, PUSH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;  // drain barrier for an aborted MMA pipeline
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int TCOLS = tmem_cols<BN>();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmP)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmQ)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  shk::pdl_wait();  // inputs of the previous kernel are complete from here on
  const uint32_t tmem_base = *tmem_slot;
  const int total_work = g.groups ? (*g.num_groups) * g.tiles_p : g.tiles_p * g.tiles_q * g.splits;
  // Dependents may launch once this CTA's last tile is accumulated (triggered by the epilogue).
  if (static_cast<int>(blockIdx.x) >= total_work) shk::pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool aborted = false;
      const uint64_t pol_p = g.p_is_weight ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_q = g.p_is_weight ? policy_evict_last() : policy_evict_first();
      for (int w = blockIdx.x; w < total_work && !aborted; w += gridDim.x) {
        const Work wk = decode_work(w, g, BN);
        const int kb0 = wk.sp * g.kb_per_split;
        const int kb1 = min(kb0 + g.kb_per_split, g.kb_total);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            if (g.err) atomicCAS(g.err, 0, 1);
            *abort_flag = 1;
            aborted = true;
            break;
          }
          mbar_expect_tx(&full[stage], S::STAGE_BYTES);
          uint8_t* sp = smem + stage * S::STAGE_BYTES;
          tma_load_2d_hint(sp, &tmP, kb * BK, wk.p_y, &full[stage], pol_p);
          tma_load_2d_hint(sp + S::P_BYTES, &tmQ, kb * BK, wk.q_y, &full[stage], pol_q);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (aborted) {
        // Every load still in flight must land before the CTA exits (bounded).
        for (int64_t i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i)
          (void)mbar_wait_drain(&full[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1));
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16(BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int w = blockIdx.x; w < total_work; w += gridDim.x) {
        const Work wk = decode_work(w, g, BN);
        const int kb0 = wk.sp * g.kb_per_split;
        const int kb1 = min(kb0 + g.kb_per_split, g.kb_total);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
          if (g.err) atomicCAS(g.err, 0, 2);
          *abort_flag = 1;
          break;
        }
        fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t sp = smem_addr(smem + stage * S::STAGE_BYTES);
          const uint32_t sq = sp + S::P_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            mma_bf16(tmem_d, sw128_desc(sp + kk * 32), sw128_desc(sq + kk * 32), IDESC,
                     (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          if (g.err) atomicCAS(g.err, 0, 3);
          *abort_flag = 1;
          // Wait (bounded) for the MMAs already issued before TMEM is freed.
          mma_commit(mma_done);
          (void)mbar_wait_drain(mma_done, 0);
          break;
        }
        mma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    const uint32_t push_par = g.push ? ((*g.push_epoch + 1u) & 1u) : 0u;
    for (int w = blockIdx.x; w < total_work; w += gridDim.x) {
      const Work wk = decode_work(w, g, BN);
      // the warp agrees on the outcome: its TMEM loads (.sync.aligned) run on all lanes or none
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, abort_flag))) {
        if (g.err && lane == 0) atomicCAS(g.err, 0, 4);
        *abort_flag = 1;
        break;
      }
      if (warp == 2 && lane == 0 && w + static_cast<int>(gridDim.x) >= total_work) shk::pdl_trigger();
      fence_after();
      const int p = wk.tp * BM + row;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;
      if constexpr (PUSH) {
        // Stage this warp's 32 rows x 64 columns in shared memory, then write
        // 128-byte row segments (16 B per lane) to the rows' owner ranks.
        __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(smem + S::PUSH_OFF) + (warp - 2) * 32 * PUSH_LD;
        const int64_t slot = (static_cast<int64_t>(push_par) * g.push_world + g.push_rank) * g.push_max_T;
#pragma unroll 1
        for (int c64 = 0; c64 < BN; c64 += 64) {
#pragma unroll 1
          for (int c = c64; c < c64 + 64; c += 16) {
            float v[16];
            __syncwarp();
            tmem_ld16(tbase + c, v);
            uint4 pk[2];
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(pk);
#pragma unroll
            for (int i = 0; i < 8; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            uint4* d = reinterpret_cast<uint4*>(stg + lane * PUSH_LD + (c - c64));
            d[0] = pk[0];
            d[1] = pk[1];
          }
          __syncwarp();
#pragma unroll 1
          for (int it = 0; it < 8; ++it) {
            const int rr = it * 4 + (lane >> 3), seg = lane & 7;
            const int pr = wk.tp * BM + quad * 32 + rr;
            const int q = wk.q_base + c64 + seg * 8;
            if (pr >= wk.p_lim || q >= wk.q_lim) continue;
            __nv_bfloat16* dst = g.push_recv[pr / g.push_rows] + (slot + pr) * g.push_n + q;
            const __nv_bfloat16* src = stg + rr * PUSH_LD + seg * 8;
            if (q + 8 <= wk.q_lim && (g.push_n & 7) == 0) {
              *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
            } else {
              for (int i = 0; i < 8 && q + i < wk.q_lim; ++i) dst[i] = src[i];
            }
          }
          __syncwarp();
        }
      }
#pragma unroll 1
      for (int c = 0; c < (PUSH ? 0 : BN); c += 16) {
        float v[16];
        __syncwarp();
        tmem_ld16(tbase + c, v);
        const int q0 = wk.q_base + c;
        if (p >= wk.p_lim) {
        } else if (PUSH) {
          // handled below per 64-column chunk
        } else if (SPLIT) {
          float* dst = g.ws + (static_cast<int64_t>(wk.sp) * g.rows_p + p) * g.rows_q + q0;
          if (q0 + 16 <= wk.q_lim && (g.rows_q & 3) == 0) {
#pragma unroll
            for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          } else {
            for (int i = 0; i < 16 && q0 + i < wk.q_lim; ++i) dst[i] = v[i];
          }
        } else if (!TRANS) {
          __nv_bfloat16* dst = g.out + static_cast<int64_t>(p) * g.ldo + q0;
          if (q0 + 16 <= wk.q_lim && (g.ldo & 7) == 0) {
            uint4 pk[2];
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(pk);
#pragma unroll
            for (int i = 0; i < 8; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            reinterpret_cast<uint4*>(dst)[0] = pk[0];
            reinterpret_cast<uint4*>(dst)[1] = pk[1];
          } else {
            for (int i = 0; i < 16 && q0 + i < wk.q_lim; ++i) dst[i] = __float2bfloat16(v[i]);
          }
        } else {
          for (int i = 0; i < 16 && q0 + i < wk.q_lim; ++i)
            g.out[static_cast<int64_t>(q0 + i) * g.ldo + p] = __float2bfloat16(v[i]);
        }
      }
      fence_before();
      mbar_arrive(&tempty[acc]);
      if (g.push) {
        // Each warp counts its own stores: the warp's lanes' stores precede the
        // arrival counts (__syncwarp + release cumulativity at system scope).
        // Non-TRANS: the warp's 32 token rows; TRANS: the tile's token columns.
        __syncwarp();
        if (lane == 0) {
          int t0, t1;
          if (!TRANS) {
            t0 = wk.tp * BM + quad * 32;
            t1 = min(t0 + 32, wk.p_lim);
          } else {
            t0 = wk.q_base;
            t1 = min(wk.q_base + BN, wk.q_lim);
          }
          for (int o = t0 / g.push_rows; t0 < t1 && o <= (t1 - 1) / g.push_rows && o < g.push_world; ++o)
            asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(g.push_cnt[o] + push_par) : "memory");
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TCOLS));
  }
}

// ============================================================================
// CTA-pair GEMM (cta_group::2).  A cluster of two CTAs on neighbouring SMs
// computes a 256 x BN tile: CTA r loads P rows [256 tp + 128 r, +128) and Q
// rows [BN tq + r BN/2, +BN/2) with its own TMA loads (no multicast); both
// loads count on the LEADER CTA's full barrier.  The leader's single MMA
// thread issues tcgen05.mma.cta_group::2 (M = 256, N = BN): the tensor cores
// of both SMs read A from their own CTA and B from both, and each CTA's TMEM
// receives its 128 rows.  Per SM and 64-wide k-block that is 16 KB of A plus
// BN/2 x 128 B of B for 128 x BN x 64 MACs -- half the B traffic of a
// one-CTA 128 x BN tile, which is what the L2 -> SM path needs at M >= 256.
//
// Barriers (all counts per phase):
//   full[s]   leader only: 1 arrive.expect_tx (both CTAs' bytes) + TMA tx
//   empty[s]  each CTA: 1 commit from the leader's MMA thread
//   tfull[a]  each CTA: 1 commit from the leader's MMA thread
//   tempty[a] leader only: 8 arrives (4 epilogue warps x 2 CTAs)
// Aborts (bounded waits) are mirrored into the peer's flag; before exit both
// CTAs give in-flight loads time to land, meet at a cluster barrier and free
// TMEM together.
// ============================================================================
constexpr int PAIR_ROWS = 128;  // P rows per CTA; the pair tile is 256 rows

// TMEM columns between the two accumulators (a power of two, so N = 192 tiles start 256-aligned).
template <int BN>
__host__ __device__ constexpr int pair_acc_cols() {
  return BN <= 128 ? 128 : 256;
}
template <int BN>
__host__ __device__ constexpr int pair_tmem_cols() {
  return 2 * pair_acc_cols<BN>();
}

template <int BN, int STAGES, bool PUSH = false>
struct PairSmem {
  static constexpr int A_BYTES = PAIR_ROWS * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int PUSH_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = PUSH_OFF + (PUSH ? PUSH_STAGE_BYTES : 0);
  static constexpr int TOTAL = BAR_OFF + (2 * STAGES + 5) * 8 + 16 + 1024;
  static_assert(B_BYTES % 1024 == 0, "B half tile must keep the 1024-byte swizzle alignment");
  static_assert(TOTAL <= 227 * 1024, "shared memory budget");
};

template <int BN, int STAGES, bool TRANS, bool SPLIT, bool PUSH = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmQ,
                     GemmParams g) {
  using S = PairSmem<BN, STAGES, PUSH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int TCOLS = pair_tmem_cols<BN>();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmP)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmQ)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before any remote arrive / complete_tx
  fence_after();
  shk::pdl_wait();  // inputs of the previous kernel are complete from here on
  const uint32_t tmem_base = *tmem_slot;
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  const int total_work = g.tiles_p * g.tiles_q * g.splits;
  // Dependents may launch once this CTA's last tile is accumulated (triggered by the epilogue).
  if (cid >= total_work) shk::pdl_trigger();
  const uint32_t peer_abort = map_to_rank(const_cast<int*>(abort_flag), rank ^ 1);
  auto raise = [&](int code) {
    if (g.err) atomicCAS(g.err, 0, code);
    *abort_flag = 1;
    st_cluster_u32(peer_abort, 1);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint64_t pol_p = g.p_is_weight ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_q = g.p_is_weight ? policy_evict_last() : policy_evict_first();
      for (int w = cid; w < total_work; w += ncl) {
        const Work wk = decode_work(w, g, BN);
        int p_y = wk.tp * (2 * PAIR_ROWS) + static_cast<int>(rank) * PAIR_ROWS;
        int q_y = wk.tq * BN + static_cast<int>(rank) * (BN / 2);
        if (p_y >= g.rows_p) p_y = 0;  // fully outside: load valid rows that are never stored
        if (q_y >= g.rows_q) q_y = 0;
        const int kb0 = wk.sp * g.kb_per_split;
        const int kb1 = min(kb0 + g.kb_per_split, g.kb_total);
        bool stop = false;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            raise(1);
            stop = true;
            break;
          }
          if (leader) mbar_expect_tx(&full[stage], 2 * S::STAGE_BYTES);
          uint8_t* sp = smem + stage * S::STAGE_BYTES;
          const uint32_t bar = map_to_rank(&full[stage], 0);
          tma_load_2d_pair_hint(sp, &tmP, kb * BK, p_y, bar, pol_p);
          tma_load_2d_pair_hint(sp + S::A_BYTES, &tmQ, kb * BK, q_y, bar, pol_q);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (stop) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_mn(2 * PAIR_ROWS, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int w = cid; w < total_work; w += ncl) {
        const Work wk = decode_work(w, g, BN);
        const int kb0 = wk.sp * g.kb_per_split;
        const int kb1 = min(kb0 + g.kb_per_split, g.kb_total);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
          raise(2);
          break;
        }
        fence_after();
        const uint32_t tmem_d = tmem_base + acc * pair_acc_cols<BN>();
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t sa = smem_addr(smem + stage * S::STAGE_BYTES);
          const uint32_t sb = sa + S::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_bf16_pair(tmem_d, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), IDESC,
                          (kb > kb0 || kk > 0) ? 1u : 0u);
          mma_commit_pair_both(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          raise(3);
          mma_commit_pair_local(mma_done);
          (void)mbar_wait_drain(mma_done, 0);
          break;
        }
        mma_commit_pair_both(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    const uint32_t push_par = PUSH ? ((*g.push_epoch + 1u) & 1u) : 0u;
    for (int w = cid; w < total_work; w += ncl) {
      const Work wk = decode_work(w, g, BN);
      // the warp agrees on the outcome: its TMEM loads (.sync.aligned) run on all lanes or none
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, abort_flag))) {
        if (lane == 0) raise(4);
        break;
      }
      if (warp == 2 && lane == 0 && w + ncl >= total_work) shk::pdl_trigger();
      fence_after();
      const int p = wk.tp * (2 * PAIR_ROWS) + static_cast<int>(rank) * PAIR_ROWS + row;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * pair_acc_cols<BN>();
      const int row0 = wk.tp * (2 * PAIR_ROWS) + static_cast<int>(rank) * PAIR_ROWS + quad * 32;
      if constexpr (PUSH) {
        // as in the one-CTA push epilogue: stage 32 rows x 64 columns, write 128-byte row segments
        __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(smem + S::PUSH_OFF) + (warp - 2) * 32 * PUSH_LD;
        const int64_t slot = (static_cast<int64_t>(push_par) * g.push_world + g.push_rank) * g.push_max_T;
#pragma unroll 1
        for (int c64 = 0; c64 < BN; c64 += 64) {
#pragma unroll 1
          for (int c = c64; c < c64 + 64; c += 16) {
            float v[16];
            __syncwarp();
            tmem_ld16(tbase + c, v);
            uint4 pk[2];
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(pk);
#pragma unroll
            for (int i = 0; i < 8; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            uint4* d = reinterpret_cast<uint4*>(stg + lane * PUSH_LD + (c - c64));
            d[0] = pk[0];
            d[1] = pk[1];
          }
          __syncwarp();
#pragma unroll 1
          for (int it = 0; it < 8; ++it) {
            const int rr = it * 4 + (lane >> 3), seg = lane & 7;
            const int pr = row0 + rr;
            const int q = wk.q_base + c64 + seg * 8;
            if (pr >= wk.p_lim || q >= wk.q_lim) continue;
            __nv_bfloat16* dst = g.push_recv[pr / g.push_rows] + (slot + pr) * g.push_n + q;
            const __nv_bfloat16* src = stg + rr * PUSH_LD + seg * 8;
            if (q + 8 <= wk.q_lim && (g.push_n & 7) == 0) {
              *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
            } else {
              for (int i = 0; i < 8 && q + i < wk.q_lim; ++i) dst[i] = src[i];
            }
          }
          __syncwarp();
        }
      }
#pragma unroll 1
      for (int c = 0; c < (PUSH ? 0 : BN); c += 16) {
        float v[16];
        __syncwarp();
        tmem_ld16(tbase + c, v);
        const int q0 = wk.q_base + c;
        if (p >= wk.p_lim) {
        } else if (SPLIT) {
          float* dst = g.ws + (static_cast<int64_t>(wk.sp) * g.rows_p + p) * g.rows_q + q0;
          if (q0 + 16 <= wk.q_lim && (g.rows_q & 3) == 0) {
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          } else {
            for (int i = 0; i < 16 && q0 + i < wk.q_lim; ++i) dst[i] = v[i];
          }
        } else if (!TRANS) {
          __nv_bfloat16* dst = g.out + static_cast<int64_t>(p) * g.ldo + q0;
          if (q0 + 16 <= wk.q_lim && (g.ldo & 7) == 0) {
            uint4 pk[2];
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(pk);
#pragma unroll
            for (int i = 0; i < 8; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            reinterpret_cast<uint4*>(dst)[0] = pk[0];
            reinterpret_cast<uint4*>(dst)[1] = pk[1];
          } else {
            for (int i = 0; i < 16 && q0 + i < wk.q_lim; ++i) dst[i] = __float2bfloat16(v[i]);
          }
        } else {
          for (int i = 0; i < 16 && q0 + i < wk.q_lim; ++i)
            g.out[static_cast<int64_t>(q0 + i) * g.ldo + p] = __float2bfloat16(v[i]);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_rank(&tempty[acc], 0));
      if constexpr (PUSH) {  // this warp's 32 token rows are stored: count them at their owners
        if (lane == 0) {
          const int t1 = min(row0 + 32, wk.p_lim);
          for (int o = row0 / g.push_rows; row0 < t1 && o <= (t1 - 1) / g.push_rows && o < g.push_world; ++o)
            asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(g.push_cnt[o] + push_par) : "memory");
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
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
  cluster_sync();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TCOLS));
  }
}

// out[(trans ? q : p)] = bf16(sum over splits of ws[s][p][q]) in fixed split order;
// four consecutive q per thread (float4 loads) when rows_q % 4 == 0.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, __nv_bfloat16* __restrict__ out, int splits,
                                     int rows_p, int rows_q, int ldo, int trans) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int64_t n = static_cast<int64_t>(rows_p) * rows_q;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if ((rows_q & 3) == 0) {
    for (int64_t i4 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i4 < n / 4; i4 += stride) {
      float4 s = reinterpret_cast<const float4*>(ws)[i4];
      for (int k = 1; k < splits; ++k) {
        const float4 v = reinterpret_cast<const float4*>(ws + k * n)[i4];
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      const int64_t i = i4 * 4;
      const int p = static_cast<int>(i / rows_q), q = static_cast<int>(i % rows_q);
      if (!trans) {
        __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(out + static_cast<int64_t>(p) * ldo + q);
        o[0] = __floats2bfloat162_rn(s.x, s.y);
        o[1] = __floats2bfloat162_rn(s.z, s.w);
      } else {
        const float v[4] = {s.x, s.y, s.z, s.w};
        for (int j = 0; j < 4; ++j) out[static_cast<int64_t>(q + j) * ldo + p] = __float2bfloat16(v[j]);
      }
    }
    return;
  }
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    float s = 0.f;
    for (int k = 0; k < splits; ++k) s += ws[k * n + i];
    const int p = static_cast<int>(i / rows_q), q = static_cast<int>(i % rows_q);
    const int64_t o = trans ? static_cast<int64_t>(q) * ldo + p : static_cast<int64_t>(p) * ldo + q;
    out[o] = __float2bfloat16(s);
  }
}

}  // namespace tc
}  // namespace shk

using namespace shk::tc;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D bf16 K-major map: dims {K, rows}, box {64, box_rows}, 128-byte swizzle.
int make_map(CUtensorMap* m, const void* base, int rows, int K, int64_t row_stride_elems, int box_rows) {
  auto enc = get_encode();
  if (!enc) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_elems * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

constexpr int kMaxDevices = 64;

// Opt a kernel into its dynamic shared-memory size once per device (the
// attribute call costs microseconds of host time on every launch otherwise).
int set_smem_once(const void* k, int bytes, bool* ready) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = 0;
  if (ready[dev]) return 0;
  const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  ready[dev] = true;
  return 0;
}

template <int BN, int STAGES, bool TRANS, bool SPLIT>
int launch_t(const CUtensorMap& mp, const CUtensorMap& mq, const GemmParams& g, int grid, cudaStream_t st) {
  using S = Smem<BN, STAGES>;
  auto k = gemm_kernel<BN, STAGES, TRANS, SPLIT>;
  static bool ready[kMaxDevices] = {false};
  const int e = set_smem_once(reinterpret_cast<const void*>(k), S::TOTAL, ready);
  if (e) return e;
  shk::launch(k, dim3(grid), dim3(192), S::TOTAL, st, mp, mq, g);
  return static_cast<int>(cudaGetLastError());
}

template <int BN, int STAGES>
int launch_push(const CUtensorMap& mp, const CUtensorMap& mq, const GemmParams& g, int grid, cudaStream_t st) {
  using S = Smem<BN, STAGES, true>;
  auto k = gemm_kernel<BN, STAGES, false, false, true>;
  static bool ready[kMaxDevices] = {false};
  const int e = set_smem_once(reinterpret_cast<const void*>(k), S::TOTAL, ready);
  if (e) return e;
  shk::launch(k, dim3(grid), dim3(192), S::TOTAL, st, mp, mq, g);
  return static_cast<int>(cudaGetLastError());
}

template <int BN, int STAGES>
int launch_bn(const CUtensorMap& mp, const CUtensorMap& mq, const GemmParams& g, int grid, bool trans, bool split,
              cudaStream_t st) {
  if (split) return trans ? launch_t<BN, STAGES, true, true>(mp, mq, g, grid, st)
                          : launch_t<BN, STAGES, false, true>(mp, mq, g, grid, st);
  return trans ? launch_t<BN, STAGES, true, false>(mp, mq, g, grid, st)
               : launch_t<BN, STAGES, false, false>(mp, mq, g, grid, st);
}

template <int BN, int STAGES, bool TRANS, bool SPLIT>
int launch_pair_t(const CUtensorMap& mp, const CUtensorMap& mq, const GemmParams& g, int grid, cudaStream_t st) {
  using S = PairSmem<BN, STAGES>;
  auto k = gemm_pair_kernel<BN, STAGES, TRANS, SPLIT>;
  static bool ready[kMaxDevices] = {false};
  const int e = set_smem_once(reinterpret_cast<const void*>(k), S::TOTAL, ready);
  if (e) return e;
  shk::launch(k, dim3(grid), dim3(192), S::TOTAL, st, mp, mq, g);
  return static_cast<int>(cudaGetLastError());
}

template <int BN, int STAGES>
int launch_pair_push(const CUtensorMap& mp, const CUtensorMap& mq, const GemmParams& g, int grid, cudaStream_t st) {
  using S = PairSmem<BN, STAGES, true>;
  auto k = gemm_pair_kernel<BN, STAGES, false, false, true>;
  static bool ready[kMaxDevices] = {false};
  const int e = set_smem_once(reinterpret_cast<const void*>(k), S::TOTAL, ready);
  if (e) return e;
  shk::launch(k, dim3(grid), dim3(192), S::TOTAL, st, mp, mq, g);
  return static_cast<int>(cudaGetLastError());
}

template <int BN, int STAGES>
int launch_pair_bn(const CUtensorMap& mp, const CUtensorMap& mq, const GemmParams& g, int grid, bool trans,
                   bool split, cudaStream_t st) {
  if (split) return trans ? launch_pair_t<BN, STAGES, true, true>(mp, mq, g, grid, st)
                          : launch_pair_t<BN, STAGES, false, true>(mp, mq, g, grid, st);
  return trans ? launch_pair_t<BN, STAGES, true, false>(mp, mq, g, grid, st)
               : launch_pair_t<BN, STAGES, false, false>(mp, mq, g, grid, st);
}

// Co-resident CTA pairs on this device for the pair kernel (cached per device).
int pair_clusters(int num_sms) {
  static int cached[16] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) return num_sms / 2;
  if (cached[dev]) return cached[dev];
  using S = PairSmem<256, 6>;
  auto k = gemm_pair_kernel<256, 6, false, false>;
  int n = num_sms / 2;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms, 1, 1);
    cfg.blockDim = dim3(192, 1, 1);
    cfg.dynamicSmemBytes = S::TOTAL;
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, k, &cfg) == cudaSuccess && c > 0) n = c < n ? c : n;
  }
  (void)cudaGetLastError();
  cached[dev] = n;
  return n;
}

}  // namespace

extern "C" int sh_gemm_bf16_tcgen05(const void* P, int rows_p, int64_t ldp, const void* Q, int rows_q, int64_t ldq,
                                    int K, void* out, int64_t ldo, int trans, int bn, int splits, float* ws,
                                    int* err, int num_sms, cudaStream_t stream) {
  if (K % BK != 0 || K <= 0) return -2;  // K must be a multiple of 64 (TMA inner box)
  if (rows_p <= 0 || rows_q <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(P) & 15) || (reinterpret_cast<uintptr_t>(Q) & 15) || (ldp * 2) % 16 ||
      (ldq * 2) % 16)
    return -3;  // TMA: 16-byte aligned bases and row strides
  if (bn != 64 && bn != 128 && bn != 256) return -4;
  splits = splits < 1 ? 1 : splits;
  const int kb_total = K / BK;
  if (splits > kb_total) splits = kb_total;
  const int kb_per_split = (kb_total + splits - 1) / splits;
  splits = (kb_total + kb_per_split - 1) / kb_per_split;
  if (splits > 1 && ws == nullptr) return -5;
  CUtensorMap mp, mq;
  int r = make_map(&mp, P, rows_p, K, ldp, BM);
  if (r) return 1000 + r;
  r = make_map(&mq, Q, rows_q, K, ldq, bn);
  if (r) return 2000 + r;
  GemmParams g{};
  g.rows_p = rows_p;
  g.rows_q = rows_q;
  g.tiles_p = (rows_p + BM - 1) / BM;
  g.tiles_q = (rows_q + bn - 1) / bn;
  g.splits = splits;
  g.kb_total = kb_total;
  g.kb_per_split = kb_per_split;
  g.out = static_cast<__nv_bfloat16*>(out);
  g.ldo = static_cast<int>(ldo);
  g.ws = ws;
  g.err = err;
  g.p_fast = trans ? 0 : 1;  // consecutive work units share the weight tile
  g.p_is_weight = trans ? 1 : 0;
  const int work = g.tiles_p * g.tiles_q * splits;
  const int grid = work < num_sms ? work : num_sms;
  const bool split = splits > 1;
  if (bn == 256)
    r = launch_bn<256, 4>(mp, mq, g, grid, trans, split, stream);
  else if (bn == 128)
    r = launch_bn<128, 6>(mp, mq, g, grid, trans, split, stream);
  else
    r = launch_bn<64, 8>(mp, mq, g, grid, trans, split, stream);
  if (r) return 3000 + r;
  if (split) {
    const int64_t n = static_cast<int64_t>(rows_p) * rows_q;
    int blocks = static_cast<int>((n / 4 + 255) / 256);
    if (blocks > 8 * num_sms) blocks = 8 * num_sms;
    if (blocks < 1) blocks = 1;
    shk::launch(splitk_reduce_kernel, dim3(blocks), dim3(256), 0, stream, ws, static_cast<__nv_bfloat16*>(out), splits, rows_p, rows_q,
                                                      static_cast<int>(ldo), trans);
    r = static_cast<int>(cudaGetLastError());
    if (r) return 4000 + r;
  }
  return 0;
}

extern "C" int sh_gemm_bf16_grouped(const void* P, int p_total_rows, int rows_p, const void* Q, int q_total, int K,
                                    void* out, int64_t ldo, const int4* groups, const int* num_groups, int max_groups,
                                    int bn, int* err, int num_sms, cudaStream_t stream) {
  if (K % BK != 0 || K <= 0) return -2;
  if (p_total_rows <= 0 || q_total <= 0 || max_groups <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(P) & 15) || (reinterpret_cast<uintptr_t>(Q) & 15)) return -3;
  if (bn != 64 && bn != 128 && bn != 256) return -4;
  CUtensorMap mp, mq;
  int r = make_map(&mp, P, p_total_rows, K, K, BM);
  if (r) return 1000 + r;
  r = make_map(&mq, Q, q_total, K, K, bn);
  if (r) return 2000 + r;
  GemmParams g{};
  g.rows_p = rows_p;
  g.rows_q = q_total;
  g.tiles_p = (rows_p + BM - 1) / BM;
  g.tiles_q = 1;
  g.splits = 1;
  g.kb_total = K / BK;
  g.kb_per_split = K / BK;
  g.out = static_cast<__nv_bfloat16*>(out);
  g.ldo = static_cast<int>(ldo);
  g.err = err;
  g.p_fast = 1;
  g.p_is_weight = 1;  // expert weights
  g.groups = groups;
  g.num_groups = num_groups;
  const int work = max_groups * g.tiles_p;
  const int grid = work < num_sms ? work : num_sms;
  if (bn == 256)
    r = launch_bn<256, 4>(mp, mq, g, grid, true, false, stream);
  else if (bn == 128)
    r = launch_bn<128, 6>(mp, mq, g, grid, true, false, stream);
  else
    r = launch_bn<64, 8>(mp, mq, g, grid, true, false, stream);
  return r ? 3000 + r : 0;
}

extern "C" int sh_gemm_bf16_pair(const void* P, int rows_p, int64_t ldp, const void* Q, int rows_q, int64_t ldq,
                                 int K, void* out, int64_t ldo, int trans, int bn, int splits, float* ws, int* err,
                                 int num_sms, cudaStream_t stream) {
  if (K % BK != 0 || K <= 0) return -2;
  if (rows_p <= 0 || rows_q <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(P) & 15) || (reinterpret_cast<uintptr_t>(Q) & 15) || (ldp * 2) % 16 ||
      (ldq * 2) % 16)
    return -3;
  if (bn != 128 && bn != 192 && bn != 256) return -4;
  splits = splits < 1 ? 1 : splits;
  const int kb_total = K / BK;
  if (splits > kb_total) splits = kb_total;
  const int kb_per_split = (kb_total + splits - 1) / splits;
  splits = (kb_total + kb_per_split - 1) / kb_per_split;
  if (splits > 1 && ws == nullptr) return -5;
  CUtensorMap mp, mq;
  int r = make_map(&mp, P, rows_p, K, ldp, PAIR_ROWS);
  if (r) return 1000 + r;
  r = make_map(&mq, Q, rows_q, K, ldq, bn / 2);
  if (r) return 2000 + r;
  GemmParams g{};
  g.rows_p = rows_p;
  g.rows_q = rows_q;
  g.tiles_p = (rows_p + 2 * PAIR_ROWS - 1) / (2 * PAIR_ROWS);
  g.tiles_q = (rows_q + bn - 1) / bn;
  g.splits = splits;
  g.kb_total = kb_total;
  g.kb_per_split = kb_per_split;
  g.out = static_cast<__nv_bfloat16*>(out);
  g.ldo = static_cast<int>(ldo);
  g.ws = ws;
  g.err = err;
  g.p_fast = trans ? 0 : 1;
  g.p_is_weight = trans ? 1 : 0;
  const int work = g.tiles_p * g.tiles_q * splits;
  const int clusters = pair_clusters(num_sms);
  const int grid = 2 * (work < clusters ? work : clusters);
  const bool split = splits > 1;
  if (bn == 256)
    r = launch_pair_bn<256, 6>(mp, mq, g, grid, trans, split, stream);
  else if (bn == 192)
    r = launch_pair_bn<192, 7>(mp, mq, g, grid, trans, split, stream);
  else
    r = launch_pair_bn<128, 8>(mp, mq, g, grid, trans, split, stream);
  if (r) return 3000 + r;
  if (split) {
    const int64_t n = static_cast<int64_t>(rows_p) * rows_q;
    int blocks = static_cast<int>((n / 4 + 255) / 256);
    if (blocks > 8 * num_sms) blocks = 8 * num_sms;
    if (blocks < 1) blocks = 1;
    shk::launch(splitk_reduce_kernel, dim3(blocks), dim3(256), 0, stream, ws, static_cast<__nv_bfloat16*>(out), splits, rows_p, rows_q,
                                                      static_cast<int>(ldo), trans);
    r = static_cast<int>(cudaGetLastError());
    if (r) return 4000 + r;
  }
  return 0;
}

extern "C" int sh_gemm_bf16_push(const void* P, int rows_p, int64_t ldp, const void* Q, int rows_q, int64_t ldq,
                                 int K, int trans, int bn, int pair, const GemmParams* push, int* err, int num_sms,
                                 cudaStream_t stream) {
  if (K % BK != 0 || K <= 0) return -2;
  if (rows_p <= 0 || rows_q <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(P) & 15) || (reinterpret_cast<uintptr_t>(Q) & 15) || (ldp * 2) % 16 ||
      (ldq * 2) % 16)
    return -3;
  if (pair ? (bn != 128 && bn != 192 && bn != 256) : (bn != 64 && bn != 128 && bn != 256)) return -4;
  if (!push || push->push_world < 1 || push->push_world > 8 || push->push_rows <= 0 || !push->push_epoch) return -6;
  if (trans) return -7;  // the push epilogue writes token rows: activations on the 128-row side
  CUtensorMap mp, mq;
  int r = make_map(&mp, P, rows_p, K, ldp, pair ? PAIR_ROWS : BM);
  if (r) return 1000 + r;
  r = make_map(&mq, Q, rows_q, K, ldq, pair ? bn / 2 : bn);
  if (r) return 2000 + r;
  GemmParams g = *push;
  g.push = 1;
  g.rows_p = rows_p;
  g.rows_q = rows_q;
  g.tiles_p = (rows_p + (pair ? 2 * PAIR_ROWS : BM) - 1) / (pair ? 2 * PAIR_ROWS : BM);
  g.tiles_q = (rows_q + bn - 1) / bn;
  g.splits = 1;
  g.kb_total = K / BK;
  g.kb_per_split = K / BK;
  g.out = nullptr;
  g.ldo = 0;
  g.ws = nullptr;
  g.err = err;
  g.p_fast = trans ? 0 : 1;
  g.p_is_weight = trans ? 1 : 0;
  g.groups = nullptr;
  g.num_groups = nullptr;
  const int work = g.tiles_p * g.tiles_q;
  if (pair) {
    const int clusters = pair_clusters(num_sms);
    const int pgrid = 2 * (work < clusters ? work : clusters);
    if (bn == 256)
      r = launch_pair_push<256, 6>(mp, mq, g, pgrid, stream);
    else if (bn == 192)
      r = launch_pair_push<192, 6>(mp, mq, g, pgrid, stream);
    else
      r = launch_pair_push<128, 8>(mp, mq, g, pgrid, stream);
    return r ? 3000 + r : 0;
  }
  const int grid = work < num_sms ? work : num_sms;
  if (bn == 256)
    r = launch_push<256, 4>(mp, mq, g, grid, stream);
  else if (bn == 128)
    r = launch_push<128, 6>(mp, mq, g, grid, stream);
  else
    r = launch_push<64, 8>(mp, mq, g, grid, stream);
  return r ? 3000 + r : 0;
}
