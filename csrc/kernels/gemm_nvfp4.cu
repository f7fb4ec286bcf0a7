// NVFP4-weight GEMM on the tcgen05 tensor cores (W4A16): out = x W^T with W in
// the ModelOpt NVFP4 layout (packed e2m1 pairs, e4m3 scale per 16 elements,
// fp32 global scale), x in bf16.
//
// The weights take the MMA's 128-row side (swap-AB: tokens are the N
// dimension).  Per 64-wide k-block the TMA producer loads the packed weight
// tile (128 rows x 32 bytes, a quarter of the bf16 bytes) and the activation
// tile; four converter warps (one weight row per thread) decode e2m1 x block
// scale into a bf16 tile written directly in the 128-byte-swizzled layout the
// UMMA shared-memory descriptor reads, fence the generic->async proxy and
// signal the MMA warp; the single MMA thread issues tcgen05.mma kind::f16 into
// TMEM and the epilogue warps apply the per-matrix global scale while
// converting to bf16.  Dense mode tiles (weight rows x tokens); grouped mode
// walks the MoE expert-group list of the bf16 grouped GEMM (entry {q_row0,
// q_rows, p_row_offset, expert}) with per-expert global scales.  Every
// mbarrier wait is bounded; on timeout the kernel records an error code,
// stops issuing work, drains and frees TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include "gemm_nvfp4.h"
#include "pdl.cuh"
#include "tcgen05_common.cuh"

namespace shk {
namespace fp4gemm {
using namespace shk::tc;

constexpr int BM = 128, BK = 64;
constexpr int THREADS = 320;  // 0 producer, 1 MMA, 2-5 epilogue, 6-9 converter

template <int BN, int STAGES>
struct Smem {
  static constexpr int PB_BYTES = BM * BK * 2;    // bf16 weight tile (converted)
  static constexpr int Q_BYTES = BN * BK * 2;     // bf16 activation tile (TMA, 128B swizzle)
  static constexpr int PK_BYTES = BM * BK / 2;    // packed weight tile (TMA)
  static constexpr int STAGE_BYTES = PB_BYTES + Q_BYTES + PK_BYTES;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  static constexpr int TOTAL = BAR_OFF + (3 * STAGES + 5) * 8 + 16 + 1024;
  static_assert(TOTAL <= 227 * 1024, "shared memory budget");
};

struct Work {
  int tp, tq;
  int p_row0;          // first weight row of the tile (global row in the stacked matrix)
  int q_y, q_lim, q_base;
  int expert;
};

__device__ __forceinline__ Work decode_work(int w, const Fp4GemmParams& g, int bn) {
  Work r;
  if (g.groups) {
    const int4 e = g.groups[w / g.tiles_p];
    r.tp = w % g.tiles_p;
    r.tq = 0;
    r.p_row0 = e.z + r.tp * BM;
    r.q_y = e.x;
    r.q_lim = e.x + e.y;
    r.q_base = e.x;
    r.expert = e.w;
    return r;
  }
  r.tq = w % g.tiles_q;
  r.tp = w / g.tiles_q;
  r.p_row0 = r.tp * BM;
  r.q_y = r.tq * bn;
  r.q_lim = g.rows_q;
  r.q_base = r.tq * bn;
  r.expert = 0;
  return r;
}

__device__ __forceinline__ float e4m3f(uint32_t b) {
  __nv_fp8_e4m3 v;
  v.__x = static_cast<__nv_fp8_storage_t>(b & 0xFF);
  return static_cast<float>(v);
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(THREADS, 1)
    fp4_gemm_kernel(const __grid_constant__ CUtensorMap tmPK, const __grid_constant__ CUtensorMap tmQ,
                    Fp4GemmParams g) {
  using S = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);  // TMA (packed + activations)
  uint64_t* conv = full + STAGES;                                   // converter done (4 warp arrivals)
  uint64_t* empty = conv + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int TCOLS = (2 * BN <= 128) ? 128 : (2 * BN <= 256 ? 256 : 512);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
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
                 "r"(TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  shk::pdl_trigger();
  shk::pdl_wait();
  const uint32_t tmem_base = *tmem_slot;
  const int total = g.groups ? (*g.num_groups) * g.tiles_p : g.tiles_p * g.tiles_q;
  const int kbn = g.K / BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool stop = false;
      for (int w = blockIdx.x; w < total && !stop; w += gridDim.x) {
        const Work wk = decode_work(w, g, BN);
        for (int kb = 0; kb < kbn; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            if (g.err) atomicCAS(g.err, 0, 21);
            *abort_flag = 1;
            stop = true;
            break;
          }
          mbar_expect_tx(&full[stage], S::PK_BYTES + S::Q_BYTES);
          uint8_t* sp = smem + stage * S::STAGE_BYTES;
          tma_load_2d(sp + S::PB_BYTES + S::Q_BYTES, &tmPK, kb * (BK / 2), wk.p_row0, &full[stage]);
          tma_load_2d(sp + S::PB_BYTES, &tmQ, kb * BK, wk.q_y, &full[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_mn(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int w = blockIdx.x; w < total; w += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
          if (g.err) atomicCAS(g.err, 0, 22);
          *abort_flag = 1;
          break;
        }
        fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < kbn; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag) || !mbar_wait(&conv[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t sp = smem_addr(smem + stage * S::STAGE_BYTES);
          const uint32_t sq = sp + S::PB_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_bf16(tmem_d, sw128_desc(sp + kk * 32), sw128_desc(sq + kk * 32), IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          if (g.err) atomicCAS(g.err, 0, 23);
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
  } else if (warp >= 6) {
    // ------------------------------------------------------------ converters: row = thread
    const int row = threadIdx.x - 6 * 32;
    const int64_t sc_ld = g.K / 16;
    int stage = 0;
    uint32_t phase = 0;
    bool stop = false;
    for (int w = blockIdx.x; w < total && !stop; w += gridDim.x) {
      const Work wk = decode_work(w, g, BN);
      const int prow = wk.p_row0 + row;
      const bool valid = prow < g.rows_total;
      const uint32_t* srow = reinterpret_cast<const uint32_t*>(g.scales + static_cast<int64_t>(valid ? prow : 0) * sc_ld);
      uint32_t sc_next = valid ? srow[0] : 0u;
      for (int kb = 0; kb < kbn; ++kb) {
        const uint32_t sc4 = sc_next;  // four e4m3 block scales of this row's 64 elements
        if (kb + 1 < kbn && valid) sc_next = srow[kb + 1];
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          if (g.err && lane == 0) atomicCAS(g.err, 0, 24);
          *abort_flag = 1;
          stop = true;
          break;
        }
        uint8_t* sp = smem + stage * S::STAGE_BYTES;
        const uint4* pk = reinterpret_cast<const uint4*>(sp + S::PB_BYTES + S::Q_BYTES + row * (BK / 2));
        const uint4 lo = pk[0], hi = pk[1];
        const uint32_t words[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        uint8_t* dst_row = sp + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // 16-byte chunk c = elements 8c .. 8c+7
          const float s = e4m3f(sc4 >> (8 * (c >> 1)));
          const uint32_t wd = words[c];
          uint32_t outw[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t byte = (wd >> (8 * i)) & 0xFF;
            const uint32_t clo = byte & 15, chi = byte >> 4;
            const float lut[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
            const float vl = (clo & 8 ? -lut[clo & 7] : lut[clo & 7]) * s;
            const float vh = (chi & 8 ? -lut[chi & 7] : lut[chi & 7]) * s;
            __nv_bfloat162 h2 = __floats2bfloat162_rn(vl, vh);
            outw[i] = *reinterpret_cast<uint32_t*>(&h2);
          }
          *reinterpret_cast<uint4*>(dst_row + ((c ^ (row & 7)) << 4)) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int w = blockIdx.x; w < total; w += gridDim.x) {
      const Work wk = decode_work(w, g, BN);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) {
        if (g.err && lane == 0) atomicCAS(g.err, 0, 25);
        *abort_flag = 1;
        break;
      }
      fence_after();
      const int p = wk.p_row0 + row;               // global weight row
      const int n = p - (g.groups ? (wk.p_row0 - wk.tp * BM) : 0);  // output column
      const bool pv = g.groups ? (wk.tp * BM + row < g.rows_p) : (p < g.rows_total);
      const float gs = g.global_scale[wk.expert];
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        __syncwarp();
        tmem_ld16(tbase + c, v);
        if (!pv) continue;
        const int q0 = wk.q_base + c;
        for (int i = 0; i < 16 && q0 + i < wk.q_lim; ++i)
          g.out[static_cast<int64_t>(q0 + i) * g.ldo + n] = __float2bfloat16(v[i] * gs);
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

}  // namespace fp4gemm
}  // namespace shk

using namespace shk::fp4gemm;

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

int map2d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, int64_t rows, int64_t cols,
          int64_t ld_elems, int box_cols, int box_rows, CUtensorMapSwizzle sw) {
  auto enc = encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_elems * esize)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

template <int BN, int STAGES>
int launch(const CUtensorMap& pk, const CUtensorMap& q, const Fp4GemmParams& g, int grid, cudaStream_t st) {
  using S = Smem<BN, STAGES>;
  auto k = fp4_gemm_kernel<BN, STAGES>;
  static bool ready[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!ready[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL);
    if (e != cudaSuccess) return static_cast<int>(e);
    ready[dev] = true;
  }
  shk::launch(k, dim3(grid), dim3(THREADS), S::TOTAL, st, pk, q, g);
  return static_cast<int>(cudaGetLastError());
}
}  // namespace

extern "C" int sh_gemm_nvfp4(Fp4GemmParams* g, const void* x, int rows_q, int64_t ldx, int bn, int num_sms,
                             cudaStream_t stream) {
  if (g->K % BK != 0 || g->K <= 0) return -2;
  if (g->rows_total <= 0 || rows_q <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(g->packed) & 15) || (reinterpret_cast<uintptr_t>(x) & 15) || (ldx * 2) % 16 ||
      (reinterpret_cast<uintptr_t>(g->scales) & 3))
    return -3;
  if (bn != 64 && bn != 128 && bn != 256) return -4;
  CUtensorMap pk, q;
  int r = map2d(&pk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g->packed, g->rows_total, g->K / 2, g->K / 2, BK / 2, BM,
                CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r) return 1000 + r;
  r = map2d(&q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, rows_q, g->K, ldx, BK, bn, CU_TENSOR_MAP_SWIZZLE_128B);
  if (r) return 2000 + r;
  g->rows_q = rows_q;
  g->tiles_p = g->groups ? (g->rows_p + BM - 1) / BM : (g->rows_total + BM - 1) / BM;
  g->tiles_q = (rows_q + bn - 1) / bn;
  const int work = g->groups ? g->max_groups * g->tiles_p : g->tiles_p * g->tiles_q;
  const int grid = work < num_sms ? work : num_sms;
  if (bn == 256)
    r = launch<256, 3>(pk, q, *g, grid, stream);
  else if (bn == 128)
    r = launch<128, 5>(pk, q, *g, grid, stream);
  else
    r = launch<64, 6>(pk, q, *g, grid, stream);
  return r ? 3000 + r : 0;
}
