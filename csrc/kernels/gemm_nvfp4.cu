// NVFP4-weight GEMM on the tcgen05 tensor cores (W4A16): out = x W^T with W in
// the ModelOpt NVFP4 layout (packed e2m1 pairs, e4m3 scale per 16 elements,
// fp32 global scale), x in bf16.
//
// The weights take the MMA's 128-row side (swap-AB: tokens are the N
// dimension).  Two shared-memory rings decouple the weight stream from the
// math: a deep ring of packed weight tiles (128 rows x 32 bytes per 64-wide
// k-block, a quarter of the bf16 bytes, plus the tile's 512 bytes of block
// scales) that the TMA producer keeps up to PSTAGES k-blocks ahead, and a
// shallow work ring of converted bf16 weight tiles + activation tiles.  Eight
// converter warps (two threads per weight row) decode e2m1 x block scale into
// the work ring in the 128-byte-swizzled layout the UMMA shared-memory
// descriptor reads, fence the generic->async proxy and signal the MMA warp
// (one converter thread also issues the slot's activation TMA); the single MMA
// thread issues tcgen05.mma kind::f16 into TMEM and the epilogue warps apply
// the per-matrix global scale while converting to bf16.  Dense mode tiles (weight rows x tokens); grouped mode
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
constexpr int CONV_WARPS = 16;
constexpr int THREADS = (6 + CONV_WARPS) * 32;  // 0 producer, 1 MMA, 2-5 epilogue, 6-21 converters (4 per row)

template <int BN, int WSTAGES, int PSTAGES_>
struct Smem {
  static constexpr int PSTAGES = PSTAGES_;        // deep ring: packed weights + scales + activations
  static constexpr int PB_BYTES = BM * BK * 2;    // bf16 weight tile (converted, work ring)
  static constexpr int Q_BYTES = BN * BK * 2;     // bf16 activation tile (TMA, 128B swizzle)
  static constexpr int PK_BYTES = BM * BK / 2;    // packed weight tile (TMA)
  static constexpr int SC_BYTES = BM * 4;         // the tile's block scales of this k-block (bulk copy)
  // deep stage: [activations | packed | scales], padded to 1024 bytes (swizzled activation tile)
  static constexpr int P_BYTES = (Q_BYTES + PK_BYTES + SC_BYTES + 1023) / 1024 * 1024;
  static constexpr int P_OFF = WSTAGES * PB_BYTES;
  static constexpr int BAR_OFF = P_OFF + PSTAGES * P_BYTES;
  static constexpr int NBARS = 2 * PSTAGES + 2 * WSTAGES + 5;
  static constexpr int TOTAL = BAR_OFF + NBARS * 8 + 16 + 1024;
  static_assert(PB_BYTES % 1024 == 0 && Q_BYTES % 1024 == 0, "swizzled tiles stay 1024-byte aligned");
  static_assert(TOTAL <= 227 * 1024, "shared memory budget");
};

struct Work {
  int tp, tq, sp, kb0, kb1;
  int p_row0;          // first weight row of the tile (global row in the stacked matrix)
  int q_y, q_lim, q_base;
  int expert;
};

__device__ __forceinline__ Work decode_work(int w, const Fp4GemmParams& g, int bn) {
  Work r;
  const int kbn = g.K / BK;
  if (g.groups) {
    r.sp = 0;
    r.kb0 = 0;
    r.kb1 = kbn;
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
  const int tiles = g.tiles_p * g.tiles_q;
  r.sp = w / tiles;
  const int tt = w % tiles;
  r.tq = tt % g.tiles_q;
  r.tp = tt / g.tiles_q;
  r.kb0 = r.sp * g.kb_per_split;
  r.kb1 = min(r.kb0 + g.kb_per_split, kbn);
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

template <int BN, int WSTAGES, int PSTAGES>
__global__ void __launch_bounds__(THREADS, 1)
    fp4_gemm_kernel(const __grid_constant__ CUtensorMap tmPK, const __grid_constant__ CUtensorMap tmQ,
                    Fp4GemmParams g) {
  using S = Smem<BN, WSTAGES, PSTAGES>;
  constexpr int PS = S::PSTAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* pfull = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);  // activations + packed + scales landed
  uint64_t* pempty = pfull + PS;                                       // MMA done with a deep slot
  uint64_t* conv = pempty + PS;                                        // converted weight tile written
  uint64_t* wempty = conv + WSTAGES;                                   // MMA done with a work slot
  uint64_t* tfull = wempty + WSTAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int TCOLS = (2 * BN <= 128) ? 128 : (2 * BN <= 256 ? 256 : 512);
  if (threadIdx.x == 0) {
    // fetch the tensor-map descriptors while the barriers and TMEM are set up
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmPK)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmQ)) : "memory");
    for (int s = 0; s < PS; ++s) {
      mbar_init(&pfull[s], 1);
      mbar_init(&pempty[s], 1);
    }
    for (int s = 0; s < WSTAGES; ++s) {
      mbar_init(&conv[s], CONV_WARPS);
      mbar_init(&wempty[s], 1);
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
  const int total = g.groups ? (*g.num_groups) * g.tiles_p : g.tiles_p * g.tiles_q * g.splits;

  if (warp == 0) {
    // ------------------------------------------------------------ packed-weight producer
    if (lane == 0) {
      int ps = 0;
      uint32_t pph = 0;
      bool stop = false;
      for (int w = blockIdx.x; w < total && !stop; w += gridDim.x) {
        const Work wk = decode_work(w, g, BN);
        for (int kb = wk.kb0; kb < wk.kb1; ++kb) {
          if (!mbar_wait(&pempty[ps], pph ^ 1, abort_flag)) {
            if (g.err) atomicCAS(g.err, 0, 21);
            *abort_flag = 1;
            stop = true;
            break;
          }
          mbar_expect_tx(&pfull[ps], S::Q_BYTES + S::PK_BYTES + S::SC_BYTES);
          uint8_t* pp = smem + S::P_OFF + ps * S::P_BYTES;
          tma_load_2d(pp, &tmQ, kb * BK, wk.q_y, &pfull[ps]);
          tma_load_2d(pp + S::Q_BYTES, &tmPK, kb * (BK / 2), wk.p_row0, &pfull[ps]);
          const uint8_t* sc_src = g.scales + (static_cast<int64_t>(kb) * g.rows_pad + wk.p_row0) * 4;
          asm volatile(
              "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                  smem_addr(pp + S::Q_BYTES + S::PK_BYTES)),
              "l"(reinterpret_cast<uint64_t>(sc_src)), "r"(S::SC_BYTES), "r"(smem_addr(&pfull[ps]))
              : "memory");
          if (++ps == PS) {
            ps = 0;
            pph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_mn(BM, BN);
      int ws = 0, ps = 0;
      uint32_t wph = 0, pph = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int w = blockIdx.x; w < total; w += gridDim.x) {
        const Work wk = decode_work(w, g, BN);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
          if (g.err) atomicCAS(g.err, 0, 22);
          *abort_flag = 1;
          break;
        }
        fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = wk.kb0; kb < wk.kb1; ++kb) {
          if (!mbar_wait(&conv[ws], wph, abort_flag) || !mbar_wait(&pfull[ps], pph, abort_flag)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t sp = smem_addr(smem + ws * S::PB_BYTES);
          const uint32_t sq = smem_addr(smem + S::P_OFF + ps * S::P_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_bf16(tmem_d, sw128_desc(sp + kk * 32), sw128_desc(sq + kk * 32), IDESC,
                     (kb > wk.kb0 || kk > 0) ? 1u : 0u);
          mma_commit(&wempty[ws]);
          mma_commit(&pempty[ps]);
          if (++ws == WSTAGES) {
            ws = 0;
            wph ^= 1;
          }
          if (++ps == PS) {
            ps = 0;
            pph ^= 1;
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
    // ------------------------------------------------------------ converters: 2 threads per weight row
    // e2m1 code (s, e1 e0 m) -> bf16 bits s<<15 | (e1 e0 m)<<6 is code_value * 2^-126 for every code
    // (exponent 0 gives the bf16 subnormal m * 2^-127); two exact bf16x2 multiplies, by 2^63 and by
    // block_scale * 2^63, restore code_value * block_scale (at most 7 significant bits: exact in bf16).
    const int ct = threadIdx.x - 6 * 32;
    // four consecutive lanes share a row (part p: elements 16p .. 16p+15 of the k-block), so a warp
    // reads 256 contiguous packed bytes and its 16-byte stores hit distinct banks per quarter-warp
    const int row = ct >> 2, part = ct & 3;
    const __nv_bfloat162 two63 = __halves2bfloat162(__float2bfloat16(9.223372036854775808e18f),
                                                    __float2bfloat16(9.223372036854775808e18f));
    int ps = 0, ws = 0;
    uint32_t pph = 0, wph = 0;
    bool stop = false;
    for (int w = blockIdx.x; w < total && !stop; w += gridDim.x) {
      const Work wk = decode_work(w, g, BN);
      for (int kb = wk.kb0; kb < wk.kb1; ++kb) {
        if (!mbar_wait(&wempty[ws], wph ^ 1, abort_flag) || !mbar_wait(&pfull[ps], pph, abort_flag)) {
          if (g.err && lane == 0) atomicCAS(g.err, 0, 24);
          *abort_flag = 1;
          stop = true;
          break;
        }
        uint8_t* wp = smem + ws * S::PB_BYTES;
        const uint8_t* pp = smem + S::P_OFF + ps * S::P_BYTES + S::Q_BYTES;  // packed tile, then its scales
        // this thread's 16 elements: one e4m3 block scale, 8 packed bytes
        const float sf = e4m3f(pp[S::PK_BYTES + row * 4 + part]) * 9.223372036854775808e18f;
        const __nv_bfloat162 scl = __halves2bfloat162(__float2bfloat16(sf), __float2bfloat16(sf));
        const uint2 pk = *reinterpret_cast<const uint2*>(pp + row * (BK / 2) + part * 8);
        uint8_t* dst_row = wp + row * 128;
#pragma unroll
        for (int c = 0; c < 2; ++c) {  // 16-byte output chunk = 8 elements = one packed word
          const uint32_t wd = c ? pk.y : pk.x;
          const uint32_t L = wd & 0x0F0F0F0Fu, Hn = (wd >> 4) & 0x0F0F0F0Fu;
          uint32_t outw[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t y = __byte_perm(L, Hn, static_cast<uint32_t>(i | ((4 + i) << 8))) & 0x000F000Fu;
            const uint32_t bits = ((y & 0x00070007u) << 6) | ((y & 0x00080008u) << 12);
            __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&bits);
            v = __hmul2(__hmul2(v, two63), scl);
            outw[i] = *reinterpret_cast<uint32_t*>(&v);
          }
          const int cc = part * 2 + c;
          *reinterpret_cast<uint4*>(dst_row + ((cc ^ (row & 7)) << 4)) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[ws]);
        if (++ps == PS) {
          ps = 0;
          pph ^= 1;
        }
        if (++ws == WSTAGES) {
          ws = 0;
          wph ^= 1;
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
      // the warp agrees on the outcome: its TMEM loads (.sync.aligned) run on all lanes or none
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, abort_flag))) {
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
        if (g.splits > 1) {
          float* dst = g.ws + (static_cast<int64_t>(wk.sp) * g.rows_q) * g.rows_total + n;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (q0 + i < wk.q_lim) dst[static_cast<int64_t>(q0 + i) * g.rows_total] = v[i] * gs;
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (q0 + i < wk.q_lim) g.out[static_cast<int64_t>(q0 + i) * g.ldo + n] = __float2bfloat16(v[i] * gs);
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
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TCOLS));
  }
}

// out[q, n] = bf16(sum over splits of ws[s][q][n]) in split order.
__global__ void split_reduce_kernel(const float* __restrict__ ws, __nv_bfloat16* __restrict__ out, int splits,
                                    int rows_q, int n, int64_t ldo) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int64_t total = static_cast<int64_t>(rows_q) * n;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < splits; ++k) s += ws[k * total + i];
    out[(i / n) * ldo + (i % n)] = __float2bfloat16(s);
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

template <int BN, int WSTAGES, int PSTAGES>
int launch(const CUtensorMap& pk, const CUtensorMap& q, const Fp4GemmParams& g, int grid, cudaStream_t st) {
  using S = Smem<BN, WSTAGES, PSTAGES>;
  auto k = fp4_gemm_kernel<BN, WSTAGES, PSTAGES>;
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

extern "C" int sh_gemm_nvfp4(Fp4GemmParams* g, const void* x, int rows_q, int64_t ldx, int bn, int splits,
                             int num_sms, cudaStream_t stream) {
  if (g->K % BK != 0 || g->K <= 0) return -2;
  if (g->rows_total <= 0 || rows_q <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(g->packed) & 15) || (reinterpret_cast<uintptr_t>(x) & 15) || (ldx * 2) % 16 ||
      (reinterpret_cast<uintptr_t>(g->scales) & 15) || g->rows_pad % 128 || g->rows_pad < g->rows_total)
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
  const int kbn = g->K / BK;
  splits = (g->groups || splits < 1) ? 1 : (splits > kbn ? kbn : splits);
  g->kb_per_split = (kbn + splits - 1) / splits;
  splits = (kbn + g->kb_per_split - 1) / g->kb_per_split;
  g->splits = splits;
  if (splits > 1 && !g->ws) return -5;
  const int work = g->groups ? g->max_groups * g->tiles_p : g->tiles_p * g->tiles_q * splits;
  const int grid = work < num_sms ? work : num_sms;
  if (bn == 256)
    r = launch<256, 3, 4>(pk, q, *g, grid, stream);
  else if (bn == 128)
    r = launch<128, 3, 7>(pk, q, *g, grid, stream);
  else
    r = launch<64, 3, 11>(pk, q, *g, grid, stream);
  if (r) return 3000 + r;
  if (splits > 1) {
    const int64_t n = static_cast<int64_t>(rows_q) * g->rows_total;
    int blocks = static_cast<int>((n + 255) / 256);
    if (blocks > 8 * num_sms) blocks = 8 * num_sms;
    shk::launch(split_reduce_kernel, dim3(blocks), dim3(256), 0, stream, g->ws, g->out, splits, rows_q, g->rows_total,
                g->ldo);
    r = static_cast<int>(cudaGetLastError());
    if (r) return 4000 + r;
  }
  return 0;
}
