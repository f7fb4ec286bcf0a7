// Stream-K BF16 linear on CTA pairs (tcgen05 cta_group::2), weights on the MMA M side.
//
//   y[j, i] = sum_k W[i, k] X[j, k]      W: [rows_w, K] weights, X: [rows_x, K] tokens, y: [rows_x, ldy]
//
// This is the decode / verify linear of the serving step (rows_x = a few
// dozen to a few hundred tokens).  The design follows from three facts:
//
// * Tile = 256 weight rows (128 per CTA of the pair) x NT tokens, with NT up to
//   512 as one or two MMAs of N = NS per 16-wide k-step (NSUB = 1 or 2).  With
//   every token of the call in one tile, each weight byte is read from HBM by
//   exactly one CTA, and each SM pulls only 128 + NT/2 operand rows per 64-wide
//   k-block for 128 x NT x 64 MACs (NT = 384: 77 MAC per byte of L2 traffic).
// * Stream-K with the split pieces first: with U tiles on G clusters, every
//   cluster owns q = U / G whole tiles, and the k-blocks of the remaining
//   r = U % G tiles are cut into one contiguous range per cluster (over the
//   first G_sk clusters), so every SM gets the same MMA work whatever the
//   tile count (no partial last wave).  Each cluster runs its split piece
//   FIRST and its whole tiles after it: a split tile is summed by the LAST
//   cluster to finish a piece of it (every piece stores its fp32 partial in a
//   fixed slot and bumps the tile's arrival counter; the piece that sees the
//   final count adds all partials in cluster order -- a fixed order, so the
//   result does not depend on timing -- and stores the tile), and that sum
//   runs on the epilogue warps while the MMA warp already works on the whole
//   tiles.  When a cluster's split range ends in a second split piece, a
//   fix-up owed for the first waits until that piece is parked: the second
//   piece's MMAs need the (single) accumulator, which only its park frees.
//   Partials of the next 32-token chunk load while the current chunk is
//   staged.  No CTA waits for another, so there is no co-residency
//   requirement.  The counter goes back to zero after each tile, so the
//   counter array stays zero between calls (after a timed-out wait, *err is
//   set and the caller must clear the counters before the next call).
// * Weights before the dependency wait: the weights do not depend on the
//   previous kernel, so under programmatic dependent launch the producer
//   fills the ring's weight halves before griddepcontrol.wait and only the
//   token halves (the previous kernel's output) wait for it.
// * Epilogue through shared memory: each thread owns one weight row (TMEM
//   lane), reads 32 token columns per tcgen05.ld and writes their bf16 values
//   into a [32][128] staging tile; one thread stores it with a TMA tensor
//   store (clipped at the tensor's bounds), so the output leaves the SM as
//   256-byte row segments.  Three staging tiles rotate, and the next chunk's
//   TMEM read is in flight while the current chunk is staged.  Split-tile partials
//   are stored as float4 ([token / 4][row][4]), so every partial store and
//   fix-up load moves 512 contiguous bytes per warp instruction.
//
// Roles (192 threads per CTA): warp 0 = TMA producer (both CTAs; both CTAs'
// bytes counted on the leader's full barrier; no multicast), warp 1 = TMEM
// allocator + MMA issuer (leader CTA only), warps 2-5 = epilogue (both CTAs,
// one 32-lane TMEM quadrant each).  Accumulators are double-buffered when two
// fit in TMEM (NT <= 256).  Every wait is bounded; on a timeout the kernel
// records an error code in *err, mirrors the abort into the peer CTA, lets
// in-flight copies land, frees TMEM and returns.
//
// Reference parity: the reference's decode linears go to its skinny-GEMM
// lane or the library GEMM (reference: suffix_hybrid/kernels/bf16_skinny.py:1-60);
// this kernel is the B200 replacement for both.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm_tcgen05.h"
#include "pdl.cuh"
#include "tcgen05_common.cuh"

namespace shk {
namespace sk {

using namespace shk::tc;

constexpr int BK = 64;        // k-block (one 128-byte swizzle row of bf16)
constexpr int ROWS = 128;     // weight rows per CTA (MMA M = 256 per pair)
constexpr int kMaxPiecesPerTile = 3;  // split pieces per split tile (the fix-up reads them all)
constexpr int STG_T = 32;              // tokens per staging tile of the TMA-store epilogue
constexpr int EPI_THREADS = 128;
constexpr int kMaxParts = 16;  // partials a fix-up may add

__host__ __device__ constexpr int pow2ceil(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

template <int NS, int NSUB>
struct Cfg {
  static constexpr int NT = NS * NSUB;                    // tokens per tile
  static constexpr int SUB_COLS = pow2ceil(NS);           // TMEM columns between sub-accumulators
  static constexpr int ACC_COLS = SUB_COLS * NSUB;        // TMEM columns of one accumulator
  static constexpr int NACC = (2 * ACC_COLS <= 512) ? 2 : 1;
  static constexpr int TCOLS = NACC * ACC_COLS;
  static constexpr int A_BYTES = ROWS * BK * 2;           // 16 KB of weight rows
  static constexpr int B_SUB_BYTES = (NS / 2) * BK * 2;   // this CTA's half of one MMA's token rows
  static constexpr int STAGE_BYTES = A_BYTES + NSUB * B_SUB_BYTES;
  static constexpr int STG_BYTES = STG_T * ROWS * 2;      // one [32][128] bf16 staging tile
  static constexpr int NSTG = 3;                          // staging tiles in flight
  static constexpr int RING = 200 * 1024;
  static constexpr int STAGES = (RING / STAGE_BYTES) > 10 ? 10 : (RING / STAGE_BYTES);
  static constexpr int STG_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = STG_OFF + NSTG * STG_BYTES;
  static constexpr int TOTAL = BAR_OFF + (2 * STAGES + 2 * NACC + 1) * 8 + 16 + 1024;
  static_assert(NS % 32 == 0 && NS >= 64 && NS <= 256, "MMA N per instruction");
  static_assert(B_SUB_BYTES % 1024 == 0, "token half-tiles keep the 1024-byte swizzle alignment");
  static_assert(TCOLS <= 512, "TMEM columns");
  static_assert(TOTAL <= 227 * 1024, "shared memory budget");
};

// Phase stamps (SkParams::stamps, [grid][64] u64 ns), for profiling the pipeline without a profiler:
//   [0] CTA start  [1] producer: first weight loads issued  [2] producer: dependency wait passed
//   [3] producer: ns waiting for free stages  [4] MMA: ns waiting for loaded stages
//   [5] MMA: ns waiting for a free accumulator  [6] epilogue: CTA end  [7] epilogue: last fix-up done
//   [8 + 4i .. 11 + 4i] segment i < 8: MMA start, MMA issue end, epilogue saw the accumulator, TMEM freed
//   [40] ns in fix-ups  [41] ns of it in the staged output stores  [42] partials summed
constexpr int kStampSlots = 64;
__device__ __forceinline__ void stamp(const SkParams& g, int slot, unsigned long long v) {
  if (g.stamps) g.stamps[blockIdx.x * kStampSlots + slot] = v;
}

// 32 consecutive TMEM columns of this thread's lane, without waiting: the
// registers are valid after the next tmem_wait_ld().
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
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// tcgen05.wait::ld that also names the 32 registers of an outstanding load as its operands, so the
// compiler cannot move their uses above the wait.
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
// 32 consecutive TMEM columns of this thread's lane (one tcgen05.ld, one wait).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  tmem_ld32_nowait(taddr, v);
  tmem_wait_ld32(v);
}

struct Seg {
  int tile, k0, k1;  // k-blocks [k0, k1) of tile `tile`
  bool whole;        // the segment covers the tile's whole K range
  bool split;        // the tile is one of the split (stream-K) tiles
};

// Split iterations: sk_iters = (U % G) * kb, cut over the first sk_clusters clusters;
// split tile j is tile (U / G) * G + j.  Range of cluster c: [c * I / Gs, (c + 1) * I / Gs).
__device__ __forceinline__ int64_t sk_start(int64_t c, const SkParams& g) {
  return c >= g.sk_clusters ? g.sk_iters : c * g.sk_iters / g.sk_clusters;
}
// The cluster whose split range holds split iteration it.
__device__ __forceinline__ int sk_cluster_of(int64_t it, const SkParams& g) {
  return static_cast<int>(((it + 1) * g.sk_clusters + g.sk_iters - 1) / g.sk_iters - 1);
}

// The segments of one cluster, in order: its split piece(s), then its whole tiles.
struct SegIter {
  int64_t sk_it, sk_end;
  int dp_next, dp_end, sk_base;
  __device__ __forceinline__ SegIter(int c, const SkParams& g) {
    sk_it = sk_start(c, g);
    sk_end = sk_start(c + 1, g);
    dp_next = c * g.q;
    dp_end = dp_next + g.q;
    sk_base = g.q * g.clusters;
  }
  __device__ __forceinline__ bool next(Seg& s, const SkParams& g) {
    if (sk_it < sk_end) {
      const int j = static_cast<int>(sk_it / g.kb);
      const int64_t t0 = static_cast<int64_t>(j) * g.kb;
      s.tile = sk_base + j;
      s.k0 = static_cast<int>(sk_it - t0);
      s.k1 = static_cast<int>((sk_end - t0) < g.kb ? (sk_end - t0) : g.kb);
      s.whole = s.k0 == 0 && s.k1 == g.kb;
      s.split = true;
      sk_it = t0 + s.k1;
      return true;
    }
    if (dp_next < dp_end) {
      s.tile = dp_next++;
      s.k0 = 0;
      s.k1 = g.kb;
      s.whole = true;
      s.split = false;
      return true;
    }
    return false;
  }
};

template <int NS, int NSUB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_sk_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   const __grid_constant__ CUtensorMap tmY, SkParams g) {
  using C = Cfg<NS, NSUB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + C::NACC;
  uint64_t* mma_done = tempty + C::NACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* bcast = const_cast<int*>(abort_flag) + 1;  // epilogue: broadcast of the arrival count

  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < C::NACC; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmY)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(C::TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before any remote arrive / complete_tx
  fence_after();
  {  // Dependents may launch once this CTA's MMAs are done (triggered by the epilogue at its last
     // segment); a CTA without work lets them launch now.
    SegIter any(blockIdx.x >> 1, g);
    Seg first;
    if (!any.next(first, g)) shk::pdl_trigger();
  }
  // griddepcontrol.wait: the producer waits after issuing its first weight loads (below); every
  // other role waits here (the epilogue writes y and the split partials, which the previous kernel
  // may still read).
  if (g.stamps && threadIdx.x == 0) stamp(g, 0, now_ns());
  if (warp != 0) shk::pdl_wait();
  const uint32_t tmem_base = *tmem_slot;
  const int cid = blockIdx.x >> 1;
  const uint32_t peer_abort = map_to_rank(const_cast<int*>(abort_flag), rank ^ 1);
  auto raise = [&](int code) {
    if (g.err) atomicCAS(g.err, 0, code);
    *abort_flag = 1;
    st_cluster_u32(peer_abort, 1);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      // Row coordinates of a tile's weight half-tile and token sub-tiles.
      auto w_row = [&](int tile) {
        const int y = (tile / g.tiles_x) * (2 * ROWS) + static_cast<int>(rank) * ROWS;
        return y < g.rows_w ? y : 0;  // wholly outside: load valid rows whose results are never stored
      };
      auto x_row = [&](int tile, int u) {
        const int y = (tile % g.tiles_x) * C::NT + u * NS + static_cast<int>(rank) * (NS / 2);
        return y < g.rows_x ? y : 0;
      };
      // Weights read by one tile only are evict-first; with several token tiles the next tile of the
      // same cluster reads the same weight rows again, so they stay (evict-last, like the tokens).
      const uint64_t pol_w = g.tiles_x == 1 ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_x = policy_evict_last();   // tokens: read by every cluster
      // 1. Before the dependency wait: the weight halves of the first STAGES k-blocks.
      int pre_tile[C::STAGES], pre_kb[C::STAGES];
      int npre = 0;
      {
        SegIter itp(cid, g);
        Seg s;
        while (npre < C::STAGES && itp.next(s, g))
          for (int kb = s.k0; kb < s.k1 && npre < C::STAGES; ++kb) {
            pre_tile[npre] = s.tile;
            pre_kb[npre] = kb;
            if (leader) mbar_expect_tx(&full[npre], 2 * C::STAGE_BYTES);
            tma_load_2d_pair_hint(smem + npre * C::STAGE_BYTES, &tmW, kb * BK, w_row(s.tile),
                                  map_to_rank(&full[npre], 0), pol_w);
            ++npre;
          }
      }
      if (g.stamps) stamp(g, 1, now_ns());
      shk::pdl_wait();  // the tokens are the previous kernel's output
      if (g.stamps) stamp(g, 2, now_ns());
      for (int i = 0; i < npre; ++i) {
        const uint32_t bar = map_to_rank(&full[i], 0);
#pragma unroll
        for (int u = 0; u < NSUB; ++u)
          tma_load_2d_pair_hint(smem + i * C::STAGE_BYTES + C::A_BYTES + u * C::B_SUB_BYTES, &tmX, pre_kb[i] * BK,
                                x_row(pre_tile[i], u), bar, pol_x);
      }
      // 2. The rest of the k-blocks, each into the next free stage.
      int stage = npre % C::STAGES;
      uint32_t phase = npre == C::STAGES ? 1u : 0u;
      int done = 0;
      unsigned long long wait_empty_ns = 0;
      SegIter it(cid, g);
      Seg s;
      bool stop = false;
      while (!stop && it.next(s, g)) {
        const int w_y = w_row(s.tile);
        int x_y[NSUB];
#pragma unroll
        for (int u = 0; u < NSUB; ++u) x_y[u] = x_row(s.tile, u);
        for (int kb = s.k0; kb < s.k1; ++kb) {
          if (done++ < npre) continue;  // issued above
          const uint64_t tw0 = g.stamps ? now_ns() : 0;
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            raise(1);
            stop = true;
            break;
          }
          if (g.stamps) wait_empty_ns += now_ns() - tw0;
          if (leader) mbar_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
          uint8_t* sp = smem + stage * C::STAGE_BYTES;
          const uint32_t bar = map_to_rank(&full[stage], 0);
          tma_load_2d_pair_hint(sp, &tmW, kb * BK, w_y, bar, pol_w);
#pragma unroll
          for (int u = 0; u < NSUB; ++u)
            tma_load_2d_pair_hint(sp + C::A_BYTES + u * C::B_SUB_BYTES, &tmX, kb * BK, x_y[u], bar, pol_x);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (g.stamps) stamp(g, 3, wait_empty_ns);
    } else {
      shk::pdl_wait();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_mn(2 * ROWS, NS);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      SegIter it(cid, g);
      Seg s;
      int seg = 0;
      unsigned long long wait_full_ns = 0, wait_acc_ns = 0;
      while (it.next(s, g)) {
        const uint64_t ta = g.stamps ? now_ns() : 0;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
          raise(2);
          break;
        }
        if (g.stamps) {
          const uint64_t t = now_ns();
          wait_acc_ns += t - ta;
          if (seg < 8) stamp(g, 8 + 4 * seg, t);
        }
        fence_after();
        const uint32_t tmem_d = tmem_base + acc * C::ACC_COLS;
        bool ok = true;
        for (int kb = s.k0; kb < s.k1; ++kb) {
          const uint64_t tf = g.stamps ? now_ns() : 0;
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          if (g.stamps) wait_full_ns += now_ns() - tf;
          fence_after();
          const uint32_t sa = smem_addr(smem + stage * C::STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
            for (int u = 0; u < NSUB; ++u)
              mma_bf16_pair(tmem_d + u * C::SUB_COLS, sw128_desc(sa + kk * 32),
                            sw128_desc(sa + C::A_BYTES + u * C::B_SUB_BYTES + kk * 32), IDESC,
                            (kb > s.k0 || kk > 0) ? 1u : 0u);
          }
          mma_commit_pair_both(&empty[stage]);
          if (++stage == C::STAGES) {
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
        if (g.stamps && seg < 8) stamp(g, 9 + 4 * seg, now_ns());
        ++seg;
        if (++acc == C::NACC) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (g.stamps) {
        stamp(g, 4, wait_full_ns);
        stamp(g, 5, wait_acc_ns);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;              // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;       // weight row within this CTA's 128
    const int et = threadIdx.x - 64;        // 0..127 within the epilogue warps
    const bool elected = et == 0;
    const int64_t slot_elems = static_cast<int64_t>(C::NT) * ROWS;
    const int first_split = static_cast<int>(sk_start(cid, g) / g.kb);  // this cluster's first split tile j
    __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(smem + C::STG_OFF);
    int chunk = 0;  // staging tiles used so far (alternating buffers)
    int acc = 0;
    uint32_t acc_phase = 0;
    int eseg = 0;
    SegIter it(cid, g);
    Seg s;
    // One 32-token chunk of this thread's weight row (v[32], fp32) -> bf16 staging tile -> TMA tensor store
    // of [32 tokens][128 weights] (clipped at the tensor's bounds).  Two staging tiles alternate.
    unsigned long long fix_store_ns = 0, fix_ns = 0, fix_parts = 0;  // stamps of the fix-ups (elected thread)
    bool in_fix = false;
    auto store_chunk = [&](const float* v, int y_w, int y_t) {
      const uint64_t ts = (g.stamps && elected && in_fix) ? now_ns() : 0;
      __nv_bfloat16* buf = stg + (chunk % C::NSTG) * (STG_T * ROWS);
      // The store issued from this buffer NSTG chunks ago has read it (at most NSTG - 1 stores still reading).
      if (elected && chunk >= C::NSTG) bulk_wait_read<C::NSTG - 1>();
      named_barrier(1, EPI_THREADS);
#pragma unroll
      for (int i = 0; i < STG_T; ++i) buf[i * ROWS + row] = __float2bfloat16_rn(v[i]);
      fence_proxy_async_smem();
      named_barrier(1, EPI_THREADS);
      if (elected) {
        if (y_w < g.rows_w && y_t < g.rows_x) tma_store_2d(&tmY, buf, y_w, y_t);
        bulk_commit();
      }
      ++chunk;
      if (ts) fix_store_ns += now_ns() - ts;
    };
    // Sums a split tile's parked partials (nparts pieces starting at cluster c_first, cluster order) and
    // stores the tile.  Run by every epilogue thread together (named barriers inside store_chunk).
    auto fixup = [&](int j, int c_first, int nparts, int y_w, int y_x0) {
      const uint64_t tf = (g.stamps && elected) ? now_ns() : 0;
      in_fix = true;
      fix_parts += nparts;
      __threadfence();  // acquire side of the counter: the other pieces' partials are visible
      if (nparts <= 2) {
        // One or two pieces: the next chunk's partials load while the current chunk is summed and
        // staged (two chunks of loads in flight per thread).  Same summation order as below.
        auto part_of = [&](int pj) {
          const int cj = c_first + pj;
          const int fj = static_cast<int>(sk_start(cj, g) / g.kb);
          return reinterpret_cast<const float4*>(
              g.ws + ((static_cast<int64_t>(cj) * 2 + rank) * 2 + (j == fj ? 0 : 1)) * slot_elems);
        };
        const float4* p0 = part_of(0);
        const float4* p1 = part_of(nparts - 1);
        const bool two = nparts == 2;
        float4 a0[8], a1[8], b0[8], b1[8];
        auto load = [&](float4* d0, float4* d1, int c) {
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) d0[i4] = __ldcg(p0 + static_cast<int64_t>(c / 4 + i4) * ROWS + row);
          if (two)
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4) d1[i4] = __ldcg(p1 + static_cast<int64_t>(c / 4 + i4) * ROWS + row);
        };
        auto sum_store = [&](float4* d0, const float4* d1, int c) {
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) {
            d0[i4].x = 0.f + d0[i4].x;
            d0[i4].y = 0.f + d0[i4].y;
            d0[i4].z = 0.f + d0[i4].z;
            d0[i4].w = 0.f + d0[i4].w;
            if (two) {
              d0[i4].x += d1[i4].x;
              d0[i4].y += d1[i4].y;
              d0[i4].z += d1[i4].z;
              d0[i4].w += d1[i4].w;
            }
          }
          store_chunk(reinterpret_cast<const float*>(d0), y_w, y_x0 + c);
        };
        load(a0, a1, 0);
#pragma unroll 1
        for (int c = 0; c < C::NT; c += 2 * STG_T) {
          load(b0, b1, c + STG_T);
          sum_store(a0, a1, c);
          if (c + 2 * STG_T < C::NT) load(a0, a1, c + 2 * STG_T);
          sum_store(b0, b1, c + STG_T);
        }
      } else {
      const float4* parts[kMaxParts];
      for (int pj = 0; pj < nparts; ++pj) {
        const int cj = c_first + pj;
        const int fj = static_cast<int>(sk_start(cj, g) / g.kb);
        parts[pj] = reinterpret_cast<const float4*>(
            g.ws + ((static_cast<int64_t>(cj) * 2 + rank) * 2 + (j == fj ? 0 : 1)) * slot_elems);
      }
#pragma unroll 1
      for (int c = 0; c < C::NT; c += STG_T) {
        // Sum the pieces in cluster order; three pieces' loads in flight at a time.
        float4 sum[8];
#pragma unroll
        for (int i4 = 0; i4 < 8; ++i4) sum[i4] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int pj = 0; pj < nparts; pj += 3) {
          float4 ld[3][8];
#pragma unroll
          for (int u = 0; u < 3; ++u)
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4)
              if (pj + u < nparts) ld[u][i4] = __ldcg(parts[pj + u] + static_cast<int64_t>(c / 4 + i4) * ROWS + row);
#pragma unroll
          for (int u = 0; u < 3; ++u)
            if (pj + u < nparts)
#pragma unroll
              for (int i4 = 0; i4 < 8; ++i4) {
                sum[i4].x += ld[u][i4].x;
                sum[i4].y += ld[u][i4].y;
                sum[i4].z += ld[u][i4].z;
                sum[i4].w += ld[u][i4].w;
              }
        }
        float v[STG_T];
#pragma unroll
        for (int i4 = 0; i4 < 8; ++i4) {
          v[4 * i4] = sum[i4].x;
          v[4 * i4 + 1] = sum[i4].y;
          v[4 * i4 + 2] = sum[i4].z;
          v[4 * i4 + 3] = sum[i4].w;
        }
        store_chunk(v, y_w, y_x0 + c);
      }
      }
      if (g.stamps && elected) {
        stamp(g, 7, now_ns());
        fix_ns += now_ns() - tf;
        stamp(g, 40, fix_ns);
        stamp(g, 41, fix_store_ns);
        stamp(g, 42, fix_parts);
      }
      in_fix = false;
    };
    struct Fix {
      int j, c_first, nparts, y_w, y_x0;
    };
    Fix pend[2];
    int npend = 0;
    while (it.next(s, g)) {
      const int tw = s.tile / g.tiles_x, tx = s.tile % g.tiles_x;
      const int y_w = tw * (2 * ROWS) + static_cast<int>(rank) * ROWS;  // output column of weight row 0
      const int y_x0 = tx * C::NT;                                        // output row of token 0
      // The epilogue warps leave together (they meet at named barriers below).
      const bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag);
      if (named_barrier_any(1, EPI_THREADS, !ok)) {
        if (elected) raise(4);
        break;
      }
      if (g.stamps && elected && eseg < 8) stamp(g, 10 + 4 * eseg, now_ns());
      if (elected) {  // the last segment's MMAs are done: the next kernel may start launching
        SegIter peek = it;
        Seg nxt;
        if (!peek.next(nxt, g)) shk::pdl_trigger();
      }
      fence_after();
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * C::ACC_COLS;
      if (s.whole) {
        // TMEM reads one chunk ahead of the staging writes (two register sets, one wait per chunk);
        // NT is a multiple of 64.
        static_assert(C::NT % (2 * STG_T) == 0, "two chunks per step");
        auto tcol = [&](int c) { return tacc + (c / NS) * C::SUB_COLS + (c % NS); };
        float va[STG_T], vb[STG_T];
        tmem_ld32(tcol(0), va);
#pragma unroll 1
        for (int c = 0; c < C::NT; c += 2 * STG_T) {
          tmem_ld32_nowait(tcol(c + STG_T), vb);
          store_chunk(va, y_w, y_x0 + c);
          tmem_wait_ld32(vb);
          if (c + 2 * STG_T < C::NT) tmem_ld32_nowait(tcol(c + 2 * STG_T), va);
          store_chunk(vb, y_w, y_x0 + c + STG_T);
          tmem_wait_ld32(va);
        }
      } else {
        // Partial tile: park this piece's fp32 sums in the cluster's slot, then
        // count it.  Slot = (cluster, rank, first split tile of the range ? 0 : 1).
        const int j = s.tile - g.q * g.clusters;  // split tile index
        float4* mine = reinterpret_cast<float4*>(
            g.ws + ((static_cast<int64_t>(cid) * 2 + rank) * 2 + (j == first_split ? 0 : 1)) * slot_elems);
        {  // TMEM reads one chunk ahead of the stores (NT is a multiple of 64)
          auto tcol = [&](int c) { return tacc + (c / NS) * C::SUB_COLS + (c % NS); };
          auto park = [&](const float* v, int c) {
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4)
              __stcg(mine + static_cast<int64_t>(c / 4 + i4) * ROWS + row,
                     make_float4(v[4 * i4], v[4 * i4 + 1], v[4 * i4 + 2], v[4 * i4 + 3]));
          };
          float va[32], vb[32];
          tmem_ld32(tcol(0), va);
#pragma unroll 1
          for (int c = 0; c < C::NT; c += 64) {
            tmem_ld32_nowait(tcol(c + 32), vb);
            park(va, c);
            tmem_wait_ld32(vb);
            if (c + 64 < C::NT) tmem_ld32_nowait(tcol(c + 64), va);
            park(vb, c + 32);
            tmem_wait_ld32(va);
          }
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_to_rank(&tempty[acc], 0));  // TMEM is free again
        if (g.stamps && elected && eseg < 8) stamp(g, 11 + 4 * eseg, now_ns());
        __threadfence();
        named_barrier(1, EPI_THREADS);
        const int c_first = sk_cluster_of(static_cast<int64_t>(j) * g.kb, g);
        if (elected) {
          const int c_last = sk_cluster_of(static_cast<int64_t>(j + 1) * g.kb - 1, g);
          int* cnt = g.cnt + s.tile * 2 + rank;
          const int old = atomicAdd(cnt, 1);
          const bool last = old == c_last - c_first;
          if (last) *cnt = 0;  // every piece has arrived: reset for the next call
          *bcast = last ? (c_last - c_first + 1) : 0;
        }
        named_barrier(1, EPI_THREADS);
        int nparts = *bcast;
        if (nparts > kMaxParts) {  // excluded by the host's cluster clamp
          if (elected) raise(5);
          nparts = 0;
        }
        if (nparts > 0) pend[npend++] = Fix{j, c_first, nparts, y_w, y_x0};
        // A last piece's fix-up waits while the next segment is another split piece: that piece's MMAs
        // need the accumulator, which only its own park frees, so the MMA would idle for the whole
        // fix-up.  Pending fix-ups run once the next segment is a whole tile (its MMAs overlap them)
        // or there is none.
        SegIter peek = it;
        Seg nxt;
        const bool more_split = peek.next(nxt, g) && nxt.split;
        if (!more_split || npend == 2) {
          for (int f = 0; f < npend; ++f) fixup(pend[f].j, pend[f].c_first, pend[f].nparts, pend[f].y_w, pend[f].y_x0);
          npend = 0;
        }
      }
      if (s.whole) {
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_to_rank(&tempty[acc], 0));
        if (g.stamps && elected && eseg < 8) stamp(g, 11 + 4 * eseg, now_ns());
      }
      ++eseg;
      if (++acc == C::NACC) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (elected) bulk_wait_all();
    if (g.stamps && elected) stamp(g, 6, now_ns());
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
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::TCOLS));
  }
}

}  // namespace sk
}  // namespace shk

namespace {

using namespace shk::sk;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// bf16 matrix [rows][cols] (row stride in elements), box {box_cols, box_rows}.
int encode(CUtensorMap* m, const void* base, int rows, int cols, int64_t stride, int box_cols, int box_rows,
           bool swizzle128) {
  auto enc = encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

constexpr int kMaxDevices = 64;

// Index of a compiled (MMA N, MMAs per k-step) variant, -1 if none.
int variant(int ns, int nsub) {
  if (nsub == 1) return ns == 64 ? 0 : ns == 128 ? 1 : ns == 192 ? 2 : ns == 256 ? 3 : -1;
  if (nsub == 2) return ns == 192 ? 4 : ns == 256 ? 5 : -1;
  return -1;
}

template <int NS, int NSUB>
int launch_sk(const CUtensorMap& mw, const CUtensorMap& mx, const CUtensorMap& my, const SkParams& g,
              cudaStream_t st) {
  using C = Cfg<NS, NSUB>;
  auto k = gemm_sk_kernel<NS, NSUB>;
  static bool ready[kMaxDevices] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = 0;
  if (!ready[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::TOTAL);
    if (e != cudaSuccess) return static_cast<int>(e);
    ready[dev] = true;
  }
  shk::launch(k, dim3(2 * g.clusters), dim3(192), C::TOTAL, st, mw, mx, my, g);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

extern "C" int sh_gemm_sk_max_clusters(int ns, int nsub) {
  static int cached[kMaxDevices][6] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  const int which = variant(ns, nsub);
  if (which < 0) return 0;
  if (cached[dev][which]) return cached[dev][which];
  int sms = 0;
  (void)cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int n = sms / 2;
  auto query = [&](auto k, int bytes) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * n, 1, 1);
    cfg.blockDim = dim3(192, 1, 1);
    cfg.dynamicSmemBytes = bytes;
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, k, &cfg) == cudaSuccess && c > 0 && c < n) n = c;
  };
  switch (which) {
    case 0: query(gemm_sk_kernel<64, 1>, Cfg<64, 1>::TOTAL); break;
    case 1: query(gemm_sk_kernel<128, 1>, Cfg<128, 1>::TOTAL); break;
    case 2: query(gemm_sk_kernel<192, 1>, Cfg<192, 1>::TOTAL); break;
    case 3: query(gemm_sk_kernel<256, 1>, Cfg<256, 1>::TOTAL); break;
    case 4: query(gemm_sk_kernel<192, 2>, Cfg<192, 2>::TOTAL); break;
    default: query(gemm_sk_kernel<256, 2>, Cfg<256, 2>::TOTAL); break;
  }
  (void)cudaGetLastError();
  cached[dev][which] = n;
  return n;
}

extern "C" int sh_gemm_sk_shape(int rows_w, int rows_x, int K, int ns, int nsub, int clusters, int64_t* tiles,
                                int64_t* ws_floats) {
  if (K % BK != 0 || K <= 0 || rows_w <= 0 || rows_x <= 0 || clusters <= 0) return -2;
  const int nt = ns * nsub;
  const int64_t t = static_cast<int64_t>((rows_w + 2 * ROWS - 1) / (2 * ROWS)) * ((rows_x + nt - 1) / nt);
  if (tiles) *tiles = t;
  if (ws_floats) *ws_floats = static_cast<int64_t>(clusters) * 2 * 2 * nt * ROWS;
  return 0;
}

extern "C" int sh_gemm_bf16_sk(const void* W, int rows_w, int64_t ldw, const void* X, int rows_x, int64_t ldx,
                               int K, void* Y, int64_t ldy, int ns, int nsub, int clusters, float* ws, int* cnt,
                               int* err, unsigned long long* stamps, cudaStream_t stream) {
  if (K % BK != 0 || K <= 0) return -2;
  if (rows_w <= 0 || rows_x <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(W) & 15) || (reinterpret_cast<uintptr_t>(X) & 15) ||
      (reinterpret_cast<uintptr_t>(Y) & 15) || (ldw * 2) % 16 || (ldx * 2) % 16 || (ldy * 2) % 16)
    return -3;  // TMA: 16-byte aligned bases and row strides
  if (clusters < 1 || !ws || !cnt) return -5;
  const int which = variant(ns, nsub);
  if (which < 0) return -4;
  const int nt = ns * nsub;
  SkParams g{};
  g.rows_w = rows_w;
  g.rows_x = rows_x;
  g.tiles_w = (rows_w + 2 * ROWS - 1) / (2 * ROWS);
  g.tiles_x = (rows_x + nt - 1) / nt;
  g.kb = K / BK;
  const int tiles = g.tiles_w * g.tiles_x;
  g.clusters = clusters;
  g.q = tiles / g.clusters;
  g.sk_iters = static_cast<int64_t>(tiles % g.clusters) * g.kb;
  // Every split range is at least ceil(kb / 15) iterations long, so a split tile of kb
  // iterations meets at most 16 ranges (the fix-up adds at most 16 partials).
  const int64_t min_range = (g.kb + kMaxParts - 2) / (kMaxParts - 1);
  int64_t gs = g.sk_iters / min_range;
  // At most kMaxPiecesPerTile pieces per split tile: the last piece's fix-up reads all of them.
  const int64_t cap = static_cast<int64_t>(tiles % g.clusters) * kMaxPiecesPerTile;
  if (gs > cap) gs = cap;
  if (gs > g.clusters) gs = g.clusters;
  if (gs < 1) gs = 1;
  g.sk_clusters = static_cast<int>(gs);
  if (g.q == 0) g.clusters = g.sk_clusters;  // fewer tiles than clusters: only the split pieces, no idle pairs
  g.ws = ws;
  g.cnt = cnt;
  g.err = err;
  g.stamps = stamps;
  g.y = static_cast<__nv_bfloat16*>(Y);
  g.ldy = ldy;
  CUtensorMap mw, mx, my;
  int r = encode(&mw, W, rows_w, K, ldw, BK, ROWS, true);
  if (r) return 1000 + r;
  r = encode(&mx, X, rows_x, K, ldx, BK, ns / 2, true);
  if (r) return 2000 + r;
  r = encode(&my, Y, rows_x, rows_w, ldy, ROWS, STG_T, false);
  if (r) return 5000 + r;
  switch (which) {
    case 0: r = launch_sk<64, 1>(mw, mx, my, g, stream); break;
    case 1: r = launch_sk<128, 1>(mw, mx, my, g, stream); break;
    case 2: r = launch_sk<192, 1>(mw, mx, my, g, stream); break;
    case 3: r = launch_sk<256, 1>(mw, mx, my, g, stream); break;
    case 4: r = launch_sk<192, 2>(mw, mx, my, g, stream); break;
    default: r = launch_sk<256, 2>(mw, mx, my, g, stream); break;
  }
  return r ? 3000 + r : 0;
}
