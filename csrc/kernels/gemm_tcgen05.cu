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
//                 counts.  No cluster multicast anywhere.
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

namespace shk {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s per wait

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false on timeout or when another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = now_ns();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
    if (now_ns() - t0 > kTimeoutNs) return false;
  }
}

__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = now_ns();
  while (!mbar_try(bar, parity))
    if (now_ns() - t0 > kTimeoutNs) return false;
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), LBO unused (1), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;             // LBO (16 B units)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;     // SBO
  d |= static_cast<uint64_t>(1) << 46;             // version
  d |= static_cast<uint64_t>(2) << 61;             // SWIZZLE_128B
  return d;
}

// Instruction descriptor: D f32, A/B bf16, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int BN>
__host__ __device__ constexpr int tmem_cols() {
  return (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
}

template <int BN, int STAGES>
struct Smem {
  static constexpr int P_BYTES = BM * BK * 2;
  static constexpr int Q_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = P_BYTES + Q_BYTES;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  static constexpr int TOTAL = BAR_OFF + (2 * STAGES + 5) * 8 + 16 + 1024;  // + alignment slack
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

template <int BN, int STAGES, bool TRANS, bool SPLIT>
__global__ void __launch_bounds__(192, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmQ, GemmParams g) {
  using S = Smem<BN, STAGES>;
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
  const uint32_t tmem_base = *tmem_slot;
  const int total_work = g.groups ? (*g.num_groups) * g.tiles_p : g.tiles_p * g.tiles_q * g.splits;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool aborted = false;
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
          tma_load_2d(sp, &tmP, kb * BK, wk.p_y, &full[stage]);
          tma_load_2d(sp + S::P_BYTES, &tmQ, kb * BK, wk.q_y, &full[stage]);
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
    for (int w = blockIdx.x; w < total_work; w += gridDim.x) {
      const Work wk = decode_work(w, g, BN);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) {
        if (g.err && lane == 0) atomicCAS(g.err, 0, 4);
        *abort_flag = 1;
        break;
      }
      fence_after();
      const int p = wk.tp * BM + row;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        __syncwarp();
        tmem_ld16(tbase + c, v);
        const int q0 = wk.q_base + c;
        if (p >= wk.p_lim) {
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

// out[(trans ? q : p)] = bf16(sum over splits of ws[s][p][q]) in fixed split order;
// four consecutive q per thread (float4 loads) when rows_q % 4 == 0.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, __nv_bfloat16* __restrict__ out, int splits,
                                     int rows_p, int rows_q, int ldo, int trans) {
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

template <int BN, int STAGES, bool TRANS, bool SPLIT>
int launch_t(const CUtensorMap& mp, const CUtensorMap& mq, const GemmParams& g, int grid, cudaStream_t st) {
  using S = Smem<BN, STAGES>;
  auto k = gemm_kernel<BN, STAGES, TRANS, SPLIT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL);
  if (e != cudaSuccess) return static_cast<int>(e);
  k<<<grid, 192, S::TOTAL, st>>>(mp, mq, g);
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
    splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(ws, static_cast<__nv_bfloat16*>(out), splits, rows_p, rows_q,
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
