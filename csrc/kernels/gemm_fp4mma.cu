// Block-scaled NVFP4 GEMM on the tcgen05 tensor cores (W4A4): both operands
// are e2m1 with one e4m3 scale per 16 elements, the MMA applies the scales
// (tcgen05.mma kind::mxf4nvf4.block_scale.block16, K = 64 per instruction)
// and accumulates fp32 in TMEM.  This is the serving math of ModelOpt NVFP4
// checkpoints (reference: suffix_hybrid/helion_kernels/nvfp4_gemm.py:1-60, the
// quantised-activation route `nvfp4_quant_act` + `nvfp4_gemm_q`), here on the
// native FP4 tensor-core path instead of a decode-to-bf16 mainloop.
//
// Roles (192 threads, one CTA per SM, persistent over work units):
//   warp 0      TMA producer: per 256-wide k-block a 128-row weight tile and a
//               bn-row activation tile (128 bytes per row, 128-byte swizzle)
//               plus both operands' 2 KB of scale chunks (bulk copies);
//   warp 1      TMEM owner and MMA issuer: copies the four 512-byte scale
//               chunks of each operand into TMEM (tcgen05.cp 32x128b.warpx4,
//               double-buffered by k-block parity), then four block-scaled
//               MMAs; commits release the smem slot / hand the accumulator on;
//   warps 2-5   epilogue: tcgen05.ld of the fp32 accumulator, times the weight
//               global scale and the token's activation scale, bf16 stores
//               (or fp32 split-K partials).
// The weights take the MMA's M side (swap-AB); tokens are the N dimension
// (bn 64 or 128).  Dense mode tiles (weight rows x tokens x K splits); grouped
// mode walks the MoE entries {q_row0, q_rows, p_row_offset, expert} and reads
// the entry's own activation scale tile.  Every mbarrier wait is bounded; a
// timeout records an error code, stops the roles, drains the tensor pipe and
// frees TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include "gemm_fp4mma.h"
#include "nvfp4_act.cuh"
#include "pdl.cuh"
#include "tcgen05_common.cuh"

namespace shk {
namespace fp4mma {
using namespace shk::tc;
using namespace shk::nvq;

constexpr int BM = 128;
constexpr int KB = 256;         // NVFP4: k elements per pipeline stage (128 bytes per row)
constexpr int ROW_BYTES = 128;  // bytes per operand row per stage (both formats)
constexpr int SF_CHUNK = 512;   // scales of 128 rows x 4 blocks
constexpr int THREADS = 192;

// Operand formats: NVFP4 (e2m1 pairs, e4m3 scale per 16, MMA K 64, four scale chunks per 256-wide stage,
// one per MMA) or MXFP8 (e4m3, ue8m0 scale per 32, MMA K 32, one scale chunk per 128-wide stage whose
// byte j of every row word serves MMA j).
template <bool FP8>
struct Fmt {
  static constexpr int KB = FP8 ? 128 : 256;
  static constexpr int CPB = FP8 ? 1 : 4;  // scale chunks per stage and operand
};

template <int BN, int STAGES, bool FP8 = false>
struct Smem {
  static constexpr int A_BYTES = BM * ROW_BYTES;
  static constexpr int B_BYTES = BN * ROW_BYTES;
  static constexpr int SF_BYTES = Fmt<FP8>::CPB * SF_CHUNK;  // one operand's scales of one k-block
  static constexpr int STAGE = A_BYTES + B_BYTES + 2 * SF_BYTES;
  static constexpr int OUT_OFF = STAGES * STAGE;  // epilogue staging tile: bf16 [BN tokens][BM columns]
  static constexpr int SC_OFF = OUT_OFF + BN * BM * 2;  // alpha_w * a_scale of the tile's tokens [BN]
  static constexpr int BAR_OFF = SC_OFF + BN * 4;
  static constexpr int NBARS = 2 * STAGES + 5;
  static constexpr int TOTAL = BAR_OFF + NBARS * 8 + 32 + 1024;
  static_assert(STAGE % 1024 == 0, "stages stay 1024-byte aligned (128-byte swizzle atoms)");
  static_assert(TOTAL <= 227 * 1024, "shared memory budget");
};

// TMEM columns: two fp32 accumulators of BN columns, then two scale buffers of
// 8 * CPB columns (A chunks at +0/+4/..., B chunks after them).
template <int BN, bool FP8 = false>
struct Tmem {
  static constexpr int SF_COL = 2 * BN;
  static constexpr int SF_BUF = 8 * Fmt<FP8>::CPB;
  static constexpr int USED = 2 * BN + 2 * SF_BUF;
  static constexpr int COLS = USED <= 128 ? 128 : (USED <= 256 ? 256 : 512);
};

__device__ __forceinline__ uint64_t sf_desc(uint32_t saddr) {
  // no-swizzle K-major descriptor over 32 rows x 16 bytes: 8-row core matrices
  // 128 bytes apart (stride byte offset); one core matrix along k.
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(128 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  return d;
}
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
// Instruction descriptor of kind::mxf4nvf4: A and B e2m1 (format 1), K-major,
// e4m3 scales (scale format 0), scale ids 0, M x N, dense K = 64.
__host__ __device__ constexpr uint32_t idesc_nvf4(int m, int n) {
  return (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}
// Instruction descriptor of kind::mxf8f6f4: A and B e4m3 (format 0), K-major, ue8m0 scales (scale
// format 1), M x N, K = 32; the scale ids (bits 4-5 for B, 29-30 for A) pick byte `sf` of the scale words.
__host__ __device__ constexpr uint32_t idesc_mxf8(int m, int n, uint32_t sf) {
  return (sf << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (1u << 23) | (static_cast<uint32_t>(m >> 4) << 24) |
         (sf << 29);
}
__device__ __forceinline__ void mma_mxf8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}
__device__ __forceinline__ void mma_nvf4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// One acq_rel atomic add at gpu scope (the split-K ticket); after a CTA barrier it publishes, by
// cumulativity, the partial-tile stores of every thread that reached the barrier.
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

struct Work {
  int tp, sp, kb0, kb1;
  int tq_tile;                 // dense: tp * tiles_q + tq (split-K ticket / workspace slot)
  int p_row0;                  // first weight row of the tile (stacked matrix)
  int q_y, q_lim, q_base;      // first activation row, row limit, first output row
  int expert;
  int sfa_tile, sfb_tile;
};

__device__ __forceinline__ Work decode_work(int w, const Fp4MmaParams& g, int bn, int nkb) {
  Work r;
  if (g.groups) {
    const int entry = w / g.tiles_p;
    const int4 e = g.groups[entry];
    r.tp = w % g.tiles_p;
    r.sp = 0;
    r.kb0 = 0;
    r.kb1 = nkb;
    r.p_row0 = e.z + r.tp * BM;
    r.q_y = e.x;
    r.q_lim = e.x + e.y;
    r.q_base = e.x;
    r.expert = e.w;
    r.sfa_tile = e.w * g.tiles_p + r.tp;
    r.sfb_tile = entry;
    r.tq_tile = 0;
    return r;
  }
  const int tiles = g.tiles_p * g.tiles_q;
  r.sp = w / tiles;
  const int tt = w % tiles;
  const int tq = tt % g.tiles_q;
  r.tp = tt / g.tiles_q;
  r.kb0 = r.sp * g.kb_per_split;
  r.kb1 = min(r.kb0 + g.kb_per_split, nkb);
  r.p_row0 = r.tp * BM;
  r.q_y = tq * bn;
  r.q_lim = g.rows_q;
  r.q_base = tq * bn;
  r.expert = 0;
  r.sfa_tile = r.tp;
  r.sfb_tile = tq;
  r.tq_tile = tt;
  return r;
}

template <int BN, int STAGES, bool FP8>
__global__ void __launch_bounds__(THREADS, 1)
    fp4mma_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  Fp4MmaParams g) {
  using S = Smem<BN, STAGES, FP8>;
  using TM = Tmem<BN, FP8>;
  constexpr int KB = Fmt<FP8>::KB;
  constexpr int CPB = Fmt<FP8>::CPB;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base derived from the shared array itself (the compiler keeps the address space)
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* epi_flag = abort_flag + 1;  // epilogue broadcast word
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t t_entry = g.stamps ? now_ns() : 0;
  if (threadIdx.x == 0) {
    // fetch the tensor-map descriptors while the barriers and TMEM are set up
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
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
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(TM::COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint64_t t_setup = g.stamps ? now_ns() : 0;
  shk::pdl_trigger();
  shk::pdl_wait();
  const uint64_t t_wait = g.stamps ? now_ns() : 0;
  unsigned long long* stamp = g.stamps ? g.stamps + static_cast<int64_t>(blockIdx.x) * 8 : nullptr;
  if (stamp && threadIdx.x == 0) {
    stamp[0] = t_setup - t_entry;
    stamp[1] = t_wait - t_setup;
  }
  const uint32_t tmem_base = *tmem_slot;
  const int nkb = (g.K + KB - 1) / KB;
  const int kc4 = nkb * CPB;  // scale chunks per tile
  const int total = g.groups ? (*g.num_groups) * g.tiles_p : g.tiles_p * g.tiles_q * g.splits;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool stop = false;
      for (int w = blockIdx.x; w < total && !stop; w += gridDim.x) {
        const Work wk = decode_work(w, g, BN, nkb);
        const uint8_t* sfa = g.w_sf + static_cast<int64_t>(wk.sfa_tile) * kc4 * SF_CHUNK;
        const uint8_t* sfb = g.x_sf + static_cast<int64_t>(wk.sfb_tile) * kc4 * SF_CHUNK;
        for (int kb = wk.kb0; kb < wk.kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
            if (g.err) atomicCAS(g.err, 0, 41);
            *abort_flag = 1;
            stop = true;
            break;
          }
          uint8_t* st = smem + s * S::STAGE;
          mbar_expect_tx(&full[s], S::STAGE);
          tma_load_2d(st, &tmA, kb * ROW_BYTES, wk.p_row0, &full[s]);
          tma_load_2d(st + S::A_BYTES, &tmB, kb * ROW_BYTES, wk.q_y, &full[s]);
          bulk_load(st + S::A_BYTES + S::B_BYTES, sfa + kb * S::SF_BYTES, S::SF_BYTES, &full[s]);
          bulk_load(st + S::A_BYTES + S::B_BYTES + S::SF_BYTES, sfb + kb * S::SF_BYTES, S::SF_BYTES, &full[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_nvf4(BM, BN);  // (NVFP4)
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      uint32_t kcount = 0;  // k-blocks issued so far: selects the scale buffer
      for (int w = blockIdx.x; w < total; w += gridDim.x) {
        const Work wk = decode_work(w, g, BN, nkb);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
          if (g.err) atomicCAS(g.err, 0, 42);
          *abort_flag = 1;
          break;
        }
        fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = wk.kb0; kb < wk.kb1; ++kb, ++kcount) {
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          if (stamp && kcount == 0) stamp[2] = now_ns() - t_wait;
          fence_after();
          const uint32_t sa = smem_addr(smem + s * S::STAGE);
          const uint32_t sb = sa + S::A_BYTES;
          const uint32_t ssfa = sb + S::B_BYTES;
          const uint32_t ssfb = ssfa + S::SF_BYTES;
          const uint32_t tsf = tmem_base + TM::SF_COL + (kcount & 1) * TM::SF_BUF;
#pragma unroll
          for (int j = 0; j < CPB; ++j) {
            tmem_cp_sf(tsf + j * 4, sf_desc(ssfa + j * SF_CHUNK));
            tmem_cp_sf(tsf + 4 * CPB + j * 4, sf_desc(ssfb + j * SF_CHUNK));
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t acc_on = (kb > wk.kb0 || j > 0) ? 1u : 0u;
            if constexpr (FP8) {
              const uint32_t byte = static_cast<uint32_t>(j) << 30;  // scale byte j of each row word
              mma_mxf8(tmem_d, sw128_desc(sa + j * 32), sw128_desc(sb + j * 32), idesc_mxf8(BM, BN, j), tsf | byte,
                       (tsf + 4) | byte, acc_on);
            } else {
              mma_nvf4(tmem_d, sw128_desc(sa + j * 32), sw128_desc(sb + j * 32), IDESC, tsf + j * 4,
                       tsf + 16 + j * 4, acc_on);
            }
          }
          mma_commit(&empty[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) {
          if (g.err) atomicCAS(g.err, 0, 43);
          *abort_flag = 1;
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
    // ------------------------------------------------------------ epilogue (warps 2-5)
    // TMEM -> alpha_w * a_scale[token] * acc -> bf16 tile staged token-major in shared memory ->
    // 16-byte stores along each token's output row.  Split-K: the fp32 partial tile goes to its
    // workspace slot; the split that arrives last on a tile (acq_rel ticket) sums all partials in
    // split order and stores the tile, then re-arms the ticket for the next launch.
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // accumulator lane = weight row of the tile
    const int et = threadIdx.x - 64;   // 0..127
    __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(smem + S::OUT_OFF);
    float* tok = reinterpret_cast<float*>(smem + S::SC_OFF);
    const int tiles = g.tiles_p * g.tiles_q;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint64_t e_wait = 0, e_part = 0, e_store = 0, e_first = 0, tq0 = 0;
    for (int w = blockIdx.x; w < total; w += gridDim.x) {
      const Work wk = decode_work(w, g, BN, nkb);
      const int nq = min(BN, wk.q_lim - wk.q_base);  // valid tokens of the tile
      if (stamp) tq0 = now_ns();
      // token scales of the tile, fetched while the mainloop runs (the previous tile's readers passed
      // the last barrier of its iteration)
      if (et < BN) tok[et] = et < nq ? g.alpha_w[wk.expert] * g.a_scale[wk.q_base + et] : 0.f;
      // one thread waits (bounded) and broadcasts, so the named barriers below never split
      if (et == 0) {
        const bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag);
        if (!ok) {
          if (g.err) atomicCAS(g.err, 0, 44);
          *abort_flag = 1;
        }
        *epi_flag = ok ? 1 : 0;
      }
      epi_sync();
      if (!*epi_flag) break;
      fence_after();
      uint64_t tq1 = 0;
      if (stamp) {
        tq1 = now_ns();
        e_wait += tq1 - tq0;
        if (!e_first) e_first = tq1 - t_wait;
      }
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;
      const int tile = wk.tq_tile;
      bool store = true;
      if (g.splits > 1) {
        // Partial tiles are stored chunk-major: 16-column chunk cc of row r at floats (cc * BM + r) * 16, so a
        // warp writes 2 KB contiguously per chunk and the reducer reads consecutive float4s across its threads.
        const int ncc = (nq + 15) >> 4;  // column chunks holding valid tokens
        float* part = g.ws + (static_cast<int64_t>(wk.sp) * tiles + tile) * (BM * BN);
#pragma unroll 1
        for (int cc = 0; cc < ncc; ++cc) {
          float v[16];
          tmem_ld16(tbase + cc * 16, v);
          float4* dst = reinterpret_cast<float4*>(part + (cc * BM + row) * 16);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
        fence_before();
        mbar_arrive(&tempty[acc]);
        epi_sync();
        if (et == 0) {
          const int old = atom_add_acq_rel(&g.counters[tile], 1);
          const int last = old == g.splits - 1;
          if (last) g.counters[tile] = 0;
          *epi_flag = last;
        }
        epi_sync();
        store = *epi_flag != 0;
        if (stamp) {
          const uint64_t t2 = now_ns();
          e_part += t2 - tq1;
          tq1 = t2;
        }
        if (store) {
          // float4 f = et + 128 j of the tile (j < 4 ncc), summed over the splits in split order; eight f per
          // round trip with up to four splits' loads in flight (32 independent loads)
          const float4* wsv = reinterpret_cast<const float4*>(g.ws + static_cast<int64_t>(tile) * (BM * BN));
          const int64_t sstride = static_cast<int64_t>(tiles) * (BM * BN) / 4;  // float4s between splits
          const int nf = ncc * 4;
#pragma unroll 1
          for (int j0 = 0; j0 < nf; j0 += 8) {
            float4 acc4[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) acc4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s0 = 0; s0 < g.splits; s0 += 4) {
              float4 t4[4][8];  // [split][f]
#pragma unroll
              for (int sp = 0; sp < 4; ++sp) {
                const int su = min(s0 + sp, g.splits - 1);  // clamped: all loads issue back to back
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  const int j = min(j0 + u, nf - 1);
                  t4[sp][u] = __ldcg(wsv + su * sstride + et + 128 * j);
                }
              }
#pragma unroll
              for (int sp = 0; sp < 4; ++sp) {
                const float m = s0 + sp < g.splits ? 1.f : 0.f;
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  acc4[u].x += m * t4[sp][u].x;
                  acc4[u].y += m * t4[sp][u].y;
                  acc4[u].z += m * t4[sp][u].z;
                  acc4[u].w += m * t4[sp][u].w;
                }
              }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              if (j0 + u >= nf) break;
              const int q = 4 * (et + 128 * (j0 + u));  // float index in the chunk-major tile
              const int cc = q >> 11, rr = (q & 2047) >> 4, col = cc * 16 + (q & 15);
              const float a4[4] = {acc4[u].x, acc4[u].y, acc4[u].z, acc4[u].w};
#pragma unroll
              for (int e = 0; e < 4; ++e) stage[(col + e) * BM + rr] = __float2bfloat16(a4[e] * tok[col + e]);
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          if (c >= nq) break;
          float v[16];
          tmem_ld16(tbase + c, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) stage[(c + i) * BM + row] = __float2bfloat16(v[i] * tok[c + i]);
        }
        fence_before();
        mbar_arrive(&tempty[acc]);
      }
      if (store) {
        epi_sync();  // the staged tile is complete
        const int n0 = g.groups ? wk.tp * BM : wk.p_row0;
        const int n_lim = g.groups ? g.rows_p : g.rows_total;
        for (int i = et; i < nq * (BM / 8); i += 128) {
          const int ql = i / (BM / 8), seg = i - ql * (BM / 8);
          const int n = n0 + seg * 8;
          if (n >= n_lim) continue;
          const __nv_bfloat16* src = stage + ql * BM + seg * 8;
          __nv_bfloat16* dst = g.out + static_cast<int64_t>(wk.q_base + ql) * g.ldo + n;
          if (g.out_vec && n + 8 <= n_lim) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
          } else {
            for (int j = 0; j < 8 && n + j < n_lim; ++j) dst[j] = src[j];
          }
        }
        epi_sync();  // the staging tile may be overwritten
      }
      if (stamp) e_store += now_ns() - tq1;
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (stamp && et == 0) {
      stamp[3] = e_first;
      stamp[4] = e_wait;
      stamp[5] = e_part;
      stamp[6] = e_store;
      stamp[7] = now_ns() - t_entry;
    }
  }
  if (*abort_flag && warp == 0 && lane == 0) {
    // loads issued before the abort complete within microseconds; give them 200 us before the CTA exits
    const uint64_t t0 = now_ns();
    while (now_ns() - t0 < 200000) {
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TM::COLS));
  }
}

// ---------------------------------------------------------------- activation quantiser
constexpr int QUANT_THREADS = 512;

// Block b (16 values) of an activation row.  SWIGLU: the row is a fused
// gate | up projection [2K] and the activation is silu(gate) * up rounded to
// bf16 (the same expression and rounding as silu_mul_bf16_kernel), so the
// SwiGLU output is quantised without being written out.
template <bool SWIGLU>
__device__ __forceinline__ void load_act(const __nv_bfloat16* xr, int K, int b, float* v) {
  if constexpr (!SWIGLU) {
    load16(xr + b * 16, v);
  } else {
    float g[16], u[16];
    load16(xr + b * 16, g);
    load16(xr + K + b * 16, u);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(g[j] / (1.f + __expf(-g[j])) * u[j]));
  }
}

// One CTA per activation row, one thread per 16-element block (looping for K > 8192).
template <bool SWIGLU>
__global__ void __launch_bounds__(QUANT_THREADS) quant_act_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, int rows, int K, const int4* __restrict__ groups,
    const int* __restrict__ num_groups, int tile_rows, float static_g, uint8_t* __restrict__ xq,
    uint8_t* __restrict__ x_sf, float* __restrict__ a_scale) {
  shk::pdl_trigger();
  shk::pdl_wait();
  __shared__ float red[QUANT_THREADS / 32];
  const int r = blockIdx.x;
  int t, slot;
  if (groups) {
    // entries are sorted by first row: the last entry starting at or before r owns it
    int lo = 0, hi = *num_groups - 1;
    if (hi < 0) return;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (groups[mid].x <= r) lo = mid;
      else hi = mid - 1;
    }
    const int4 e = groups[lo];
    if (r < e.x || r >= e.x + e.y) return;
    t = lo;
    slot = r - e.x;
  } else {
    t = r / tile_rows;
    slot = r - t * tile_rows;
  }
  const __nv_bfloat16* xr = x + static_cast<int64_t>(r) * ldx;
  const int nblk = K / 16;
  const int kc4 = ((K + KB - 1) / KB) * 4;
  float g = static_g;
  if (!(g > 0.f)) {
    float amax = 0.f;
    for (int b = threadIdx.x; b < nblk; b += blockDim.x) {
      float v[16];
      load_act<SWIGLU>(xr, K, b, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = 0.f;
    for (int i = 0; i < static_cast<int>((blockDim.x + 31) >> 5); ++i) amax = fmaxf(amax, red[i]);
    g = row_g(amax);
  }
  const float g6 = __fdiv_rn(g, 6.f);
  if (threadIdx.x == 0) a_scale[r] = __fdiv_rn(1.f, g);
  uint8_t* sf = x_sf + static_cast<int64_t>(t) * kc4 * SF_CHUNK + (slot & 31) * 16 + ((slot >> 5) & 3) * 4;
  uint8_t* q = xq + static_cast<int64_t>(r) * (K / 2);
  for (int b = threadIdx.x; b < kc4 * 4; b += blockDim.x) {
    uint8_t s8 = 0;
    if (b < nblk) {
      float v[16];
      load_act<SWIGLU>(xr, K, b, v);
      s8 = quant16(v, g, g6, q + b * 8);
    }
    sf[(b >> 2) * SF_CHUNK + (b & 3)] = s8;
  }
}

// Rows already quantised to NVFP4 in the linear layout (codes [rows][K/2],
// e4m3 scales [rows][K/16], a_scale [rows], as the quantising expert-parallel
// dispatch sends them) gathered into the grouped W4A4 GEMM's operand layout:
// row r of group entry e takes source row token[r]; its scales land in the
// entry's scale tile exactly where quant_act_kernel puts them.
__global__ void __launch_bounds__(256) gather_nvfp4_kernel(const uint8_t* __restrict__ codes,
                                                           const uint8_t* __restrict__ scales,
                                                           const float* __restrict__ ascale,
                                                           const int* __restrict__ token, int K,
                                                           const int4* __restrict__ groups,
                                                           const int* __restrict__ num_groups, uint8_t* __restrict__ xq,
                                                           uint8_t* __restrict__ x_sf, float* __restrict__ a_scale) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int r = blockIdx.x;
  int lo = 0, hi = *num_groups - 1;
  if (hi < 0) return;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (groups[mid].x <= r) lo = mid;
    else hi = mid - 1;
  }
  const int4 e = groups[lo];
  if (r < e.x || r >= e.x + e.y) return;
  const int slot = r - e.x;
  const int64_t src = token[r];
  const uint4* s4 = reinterpret_cast<const uint4*>(codes + src * (K / 2));
  uint4* d4 = reinterpret_cast<uint4*>(xq + static_cast<int64_t>(r) * (K / 2));
  for (int i = threadIdx.x; i < K / 32; i += blockDim.x) d4[i] = s4[i];
  if (threadIdx.x == 0) a_scale[r] = ascale[src];
  const int nblk = K / 16, kc4 = ((K + KB - 1) / KB) * 4;
  uint8_t* sf = x_sf + static_cast<int64_t>(lo) * kc4 * SF_CHUNK + (slot & 31) * 16 + ((slot >> 5) & 3) * 4;
  const uint8_t* ss = scales + src * nblk;
  for (int b = threadIdx.x; b < kc4 * 4; b += blockDim.x) sf[(b >> 2) * SF_CHUNK + (b & 3)] = b < nblk ? ss[b] : 0;
}

// MXFP8 activations: per 32 values s = 2^e (ue8m0 byte e + 127) with e the smallest exponent that keeps
// amax / s <= 448, code = e4m3(x / s) (exact scaling, round to nearest even); a_scale = 1.
__global__ void __launch_bounds__(QUANT_THREADS) quant_act_mx8_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, int rows, int K, const int4* __restrict__ groups,
    const int* __restrict__ num_groups, int tile_rows, uint8_t* __restrict__ xq, uint8_t* __restrict__ x_sf,
    float* __restrict__ a_scale) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int r = blockIdx.x;
  int t, slot;
  if (groups) {
    int lo = 0, hi = *num_groups - 1;
    if (hi < 0) return;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (groups[mid].x <= r) lo = mid;
      else hi = mid - 1;
    }
    const int4 e = groups[lo];
    if (r < e.x || r >= e.x + e.y) return;
    t = lo;
    slot = r - e.x;
  } else {
    t = r / tile_rows;
    slot = r - t * tile_rows;
  }
  const __nv_bfloat16* xr = x + static_cast<int64_t>(r) * ldx;
  const int nblk = K / 32;
  const int chunks = K / 128;
  if (threadIdx.x == 0) a_scale[r] = 1.f;
  uint8_t* sf = x_sf + static_cast<int64_t>(t) * chunks * SF_CHUNK + (slot & 31) * 16 + ((slot >> 5) & 3) * 4;
  uint8_t* q = xq + static_cast<int64_t>(r) * K;
  for (int b = threadIdx.x; b < nblk; b += blockDim.x) {
    float v[32];
    load16(xr + b * 32, v);
    load16(xr + b * 32 + 16, v + 16);
    float am = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) am = fmaxf(am, fabsf(v[j]));
    int e = -127;
    if (am > 0.f) {
      int ex;
      const float m = frexpf(am / 448.f, &ex);  // am / 448 = m * 2^ex, m in [0.5, 1)
      e = (m == 0.5f) ? ex - 1 : ex;             // smallest e with am / 2^e <= 448
      e = max(-127, min(127, e));
    }
    const float inv = ldexpf(1.f, -e);
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t word = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_fp8_e4m3 c(v[4 * j + i] * inv);
        word |= static_cast<uint32_t>(c.__x) << (8 * i);
      }
      w[j] = word;
    }
    *reinterpret_cast<uint4*>(q + b * 32) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(q + b * 32 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
    sf[(b >> 2) * SF_CHUNK + (b & 3)] = static_cast<uint8_t>(e + 127);
  }
}

}  // namespace fp4mma
}  // namespace shk

using namespace shk::fp4mma;

namespace {
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

// uint8 [rows, cols] row-major, box {128 bytes, box_rows}, 128-byte swizzle.
int map_u8(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows) {
  auto enc = encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(ROW_BYTES), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

template <int BN, int STAGES, bool FP8>
int launch(const CUtensorMap& a, const CUtensorMap& b, const Fp4MmaParams& g, int grid, cudaStream_t st) {
  using S = Smem<BN, STAGES, FP8>;
  auto k = fp4mma_kernel<BN, STAGES, FP8>;
  static bool ready[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!ready[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL);
    if (e != cudaSuccess) return static_cast<int>(e);
    ready[dev] = true;
  }
  shk::launch(k, dim3(grid), dim3(THREADS), S::TOTAL, st, a, b, g);
  return static_cast<int>(cudaGetLastError());
}
}  // namespace

extern "C" int sh_nvfp4_quant_act(const void* x, int64_t ldx, int rows, int K, const int4* groups,
                                  const int* num_groups, int max_tiles, int tile_rows, float static_g, uint8_t* xq,
                                  uint8_t* x_sf, float* a_scale, int swiglu, cudaStream_t stream) {
  if (K % 64 != 0 || K <= 0 || tile_rows <= 0 || tile_rows > 128) return -2;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx * 2) % 16 || (reinterpret_cast<uintptr_t>(xq) & 7)) return -3;
  if (rows <= 0 || max_tiles <= 0) return 0;
  const int nb = ((K + KB - 1) / KB) * 4 * 4;
  const int threads = nb >= QUANT_THREADS ? QUANT_THREADS : (nb + 31) / 32 * 32;
  if (swiglu && ldx < 2 * static_cast<int64_t>(K)) return -5;
  shk::launch(swiglu ? quant_act_kernel<true> : quant_act_kernel<false>, dim3(rows), dim3(threads), 0, stream,
              static_cast<const __nv_bfloat16*>(x), ldx, rows, K, groups, num_groups, tile_rows, static_g, xq, x_sf,
              a_scale);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_nvfp4_gather_act(const uint8_t* codes, const uint8_t* scales, const float* ascale, const int* token,
                                   int rows, int K, const int4* groups, const int* num_groups, uint8_t* xq,
                                   uint8_t* x_sf, float* a_scale, cudaStream_t stream) {
  if (K % 64 != 0 || K <= 0 || !groups || !num_groups) return -2;
  if ((reinterpret_cast<uintptr_t>(codes) & 15) || (reinterpret_cast<uintptr_t>(xq) & 15)) return -3;
  if (rows <= 0) return 0;
  shk::launch(gather_nvfp4_kernel, dim3(rows), dim3(256), 0, stream, codes, scales, ascale, token, K, groups,
              num_groups, xq, x_sf, a_scale);
  return static_cast<int>(cudaGetLastError());
}

namespace {
template <bool FP8>
int run_blockscaled(Fp4MmaParams* g, const void* xq, int rows_q, int bn, int splits, int num_sms,
                    cudaStream_t stream) {
  constexpr int KBF = Fmt<FP8>::KB;
  const int row_bytes = FP8 ? g->K : g->K / 2;
  if (g->K <= 0 || g->K % (FP8 ? 128 : 64) != 0) return -2;
  if (g->rows_total <= 0 || rows_q <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(g->w) & 15) || (reinterpret_cast<uintptr_t>(xq) & 15) ||
      (reinterpret_cast<uintptr_t>(g->w_sf) & 15) || (reinterpret_cast<uintptr_t>(g->x_sf) & 15) ||
      row_bytes % 16 != 0)
    return -3;
  if (bn != 64 && bn != 128) return -4;
  CUtensorMap a, b;
  int r = map_u8(&a, g->w, g->rows_total, row_bytes, BM);
  if (r) return 1000 + r;
  r = map_u8(&b, xq, rows_q, row_bytes, bn);
  if (r) return 2000 + r;
  g->rows_q = rows_q;
  if (!g->groups) g->rows_p = g->rows_total;
  g->tiles_p = (g->rows_p + BM - 1) / BM;
  g->tiles_q = (rows_q + bn - 1) / bn;
  const int nkb = (g->K + KBF - 1) / KBF;
  splits = (g->groups || splits < 1) ? 1 : (splits > nkb ? nkb : splits);
  g->kb_per_split = (nkb + splits - 1) / splits;
  splits = (nkb + g->kb_per_split - 1) / g->kb_per_split;
  g->splits = splits;
  if (splits > 1 && (!g->ws || !g->counters)) return -5;
  g->out_vec = (g->ldo % 8 == 0) && (reinterpret_cast<uintptr_t>(g->out) % 16 == 0);
  const int work = g->groups ? g->max_groups * g->tiles_p : g->tiles_p * g->tiles_q * splits;
  const int grid = work < num_sms ? work : num_sms;
  r = bn == 128 ? launch<128, 5, FP8>(a, b, *g, grid, stream) : launch<64, 7, FP8>(a, b, *g, grid, stream);
  if (r) return 3000 + r;
  return 0;
}
}  // namespace

extern "C" int sh_gemm_fp4mma(Fp4MmaParams* g, const void* xq, int rows_q, int bn, int splits, int num_sms,
                              cudaStream_t stream) {
  return run_blockscaled<false>(g, xq, rows_q, bn, splits, num_sms, stream);
}

extern "C" int sh_gemm_mxfp8(Fp4MmaParams* g, const void* xq, int rows_q, int bn, int splits, int num_sms,
                             cudaStream_t stream) {
  return run_blockscaled<true>(g, xq, rows_q, bn, splits, num_sms, stream);
}

extern "C" int sh_mxfp8_quant_act(const void* x, int64_t ldx, int rows, int K, const int4* groups,
                                  const int* num_groups, int tile_rows, uint8_t* xq, uint8_t* x_sf, float* a_scale,
                                  cudaStream_t stream) {
  if (K % 128 != 0 || K <= 0 || tile_rows <= 0 || tile_rows > 128) return -2;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx * 2) % 16 || (reinterpret_cast<uintptr_t>(xq) & 15)) return -3;
  if (rows <= 0) return 0;
  const int nb = K / 32;
  const int threads = nb >= QUANT_THREADS ? QUANT_THREADS : (nb + 31) / 32 * 32;
  shk::launch(quant_act_mx8_kernel, dim3(rows), dim3(threads), 0, stream, static_cast<const __nv_bfloat16*>(x), ldx,
              rows, K, groups, num_groups, tile_rows, xq, x_sf, a_scale);
  return static_cast<int>(cudaGetLastError());
}
