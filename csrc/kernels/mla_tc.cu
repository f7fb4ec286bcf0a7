// Sparse / dense MLA decode on the 5th-generation tensor cores (sm_100a).
//
//   o[t, h, :] = softmax_k(q[t, h] . c[k] * scale) c[k, :V]     (absorbed form)
//
// q[t, h] is the absorbed query [q_nope W_UK | rotated q_pe] (C = 576 =
// kv_lora 512 + rope 64); a key's cache row c[k] is [normalised c_kv | rotated
// k_pe] and its value is the first V = 512 columns of the same row.  Keys are a
// token's DSA top-k positions (sparse) or every position up to the token's own
// (dense causal).
//
// Work unit (one CTA): one query token x 128 heads (the MMA M side) x one half
// of the value columns (256) x one key split.  The two value halves of a unit
// run as two CTAs that both compute S = Q K^T: O for all 512 columns would fill
// the 512 TMEM columns on its own, and the halves need no exchange.
//
// Memory plan.  Q's first 5 slabs of 64 dims live in shared memory (80 KB,
// 128-byte swizzle, one TMA load each) and its last 4 slabs in TMEM (128
// columns, written once by the softmax warps), which leaves room for a 4-stage
// ring of 32-key tiles (36 KB each).  TMEM: O [0, 256), S [256, 320) (two
// buffers), P [320, 352) (two buffers, bf16 pairs), Q [352, 480).
//
// Roles (416 threads):
//   warps 0, 6-12 producers: each computes the tile's 32 cache rows (top-k
//                 position -> block table) and issues an eighth of the tile's
//                 72 warp-wide 16-byte cp.async copies (4 keys x one 128-byte
//                 row of a 64-dim slab each), stored at the swizzled positions
//                 the MMA descriptors expect; every lane's arrival on the
//                 tile's barrier fires when its copies land;
//   warp 1        MMA issuer: S_j = Q K_j^T (M 128 x N 32 x K 576: 20 MMAs
//                 with Q from shared memory, 16 with Q from TMEM) into one of
//                 two S buffers, then O += P_{j-1} V_{j-1} (M 128 x N 256 x
//                 K 32) with P read from TMEM and V from the same key tile
//                 read MN-major, so S_{j+1} runs while tile j's softmax runs;
//   warps 2-5     softmax / epilogue, one head row per thread (a TMEM lane):
//                 read S_j, mask, online softmax in the exp2 domain, write P_j
//                 (bf16) into TMEM.  O is rescaled (TMEM load / multiply /
//                 store) only when a row's running maximum grows by more than
//                 8 (2^8), otherwise the stale maximum is kept: the final 1 / l
//                 uses the same maximum, so the result is exact.  At the end
//                 O / l leaves TMEM for the output (or the split partial and
//                 its (max, sum) for the split-order merge in mla.cu).
// Every wait is bounded (2 s): a timed-out wait records 500 + phase in *err,
// raises the CTA's abort flag, and the CTA drains its MMAs and copies in flight
// and frees its TMEM before it returns.  The one TMA load (Q) reads this GPU's
// memory without multicast.
//
// NVFP4 latent cache (352-byte rows: e2m1 pairs, e4m3 rope, permuted e4m3
// scales per 16 values): the producers load a key's packed row with 16-, 8- and
// 4-byte loads, decode each block and the rope into bf16 chunks of the swizzled
// tile in registers (exact), then fence the shared-memory writes to the tensor
// cores before they arrive; no staging buffer is needed.
//
// Reference parity: the reference's sparse MLA decode over its FP8 / NVFP4
// caches (reference: kernels-oxide/nvfp4_ds_mla/src/main.rs:1-45) computes the
// same absorbed attention over the bf16 or NVFP4 latent cache.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "mla.h"
#include "pdl.cuh"
#include "tcgen05_common.cuh"

namespace shk {
namespace mlatc {

using namespace shk::tc;

constexpr int C = 576;              // query / key row: 512 latent + 64 rope
constexpr int VH = 256;             // value columns per CTA (half of 512)
constexpr int ROWS = 128;           // heads per unit (MMA M)
constexpr int KT = 32;              // keys per tile
constexpr int SLABS = C / 64;       // 9 slabs of 64 dims (one 128-byte swizzle row each)
constexpr int QS = 5;               // Q slabs in shared memory; slabs QS.. live in TMEM
constexpr int Q_SLAB = ROWS * 128;  // 16 KB
constexpr int K_SLAB = KT * 128;    // 4 KB
constexpr int K_BYTES = SLABS * K_SLAB;  // 36 KB per key tile
constexpr int STAGES = 4;
constexpr int PROD_WARPS = 8;       // warps 0, 6-12
constexpr int THREADS = 416;
constexpr int COPIES = SLABS * (KT / 4);  // warp-wide 16-byte copies per tile (72)
constexpr int COPIES_PER_WARP = COPIES / PROD_WARPS;
static_assert(COPIES % PROD_WARPS == 0, "copies split evenly over the producer warps");
constexpr uint32_t T_O = 0, T_S = 256, T_P = 320, T_Q = 352, T_COLS = 512;
// NVFP4 latent row (kv_lora 512 + rope 64, mla.h): 256 bytes of e2m1 pairs (low nibble first), the 64 rope
// values as e4m3, 32 e4m3 scales (one per 16 values; block s at byte 8 (s % 4) + s / 4); 352 bytes.
constexpr int kFp4Rope = 256, kFp4Scales = 320, kFp4Row = 352;

struct Smem {
  static constexpr int Q = 0;
  static constexpr int K = Q + QS * Q_SLAB;            // 80 KB
  static constexpr int VALID = K + STAGES * K_BYTES;   // [STAGES] key-validity masks
  static constexpr int BAR = VALID + 64;
  static constexpr int NBAR = 2 + 2 * STAGES + 2 + 2 + 3;  // qfull, qtm, kfull, kempty, sfull, pfull, odone, drain, pv
  static constexpr int MISC = BAR + NBAR * 8;
  static constexpr int TOTAL = MISC + 64 + 1024;       // + alignment slack
};
static_assert(Smem::TOTAL <= 227 * 1024, "shared memory budget");
static_assert(Smem::K % 1024 == 0 && K_BYTES % 1024 == 0, "swizzle atoms stay 1024-byte aligned");

// MN-major 128-byte-swizzled operand: rows of 64 MN elements (128 B) along K, 8-row atoms SBO bytes
// apart along K, 64-element MN chunks LBO bytes apart.
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // version
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}
// kind::f16 instruction descriptor: D f32, A/B bf16, A K-major, B K- or MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn_major ? (1u << 16) : 0u) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}
// D (TMEM) += A (TMEM) x B (shared memory).
__device__ __forceinline__ void mma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}
// 32 consecutive TMEM columns of this thread's lane <- v (then waits for the stores).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// 8 e2m1 codes (nibble k = value k) -> 4 bf16 pairs times the block scale.  Byte-permute tables give the
// two bytes of each magnitude's bf16 encoding (0, 0.5, 1, 1.5, 2, 3, 4, 6), the code's bit 3 becomes the
// sign, and one bf16x2 multiply applies the scale (exact: at most 5 significant bits).
__device__ __forceinline__ void e2m1x8_to_bf16(uint32_t w, __nv_bfloat162 s2, uint32_t* out) {
  constexpr uint32_t kLo0 = 0xC0800000u, kLo1 = 0xC0804000u;  // low bytes of codes 0-3, 4-7
  constexpr uint32_t kHi0 = 0x3F3F3F00u, kHi1 = 0x40404040u;  // high bytes of codes 0-3, 4-7
  const uint32_t mag = w & 0x77777777u;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t sel = (mag >> (16 * h)) & 0xFFFFu;
    const uint32_t lo = __byte_perm(kLo0, kLo1, sel), hi = __byte_perm(kHi0, kHi1, sel);
    const uint32_t sg = (w >> (16 * h)) & 0x8888u;
    const uint32_t p01 = __byte_perm(lo, hi, 0x5140) | ((sg & 0x8u) << 12) | ((sg & 0x80u) << 24);
    const uint32_t p23 = __byte_perm(lo, hi, 0x7362) | ((sg & 0x800u) << 4) | ((sg & 0x8000u) << 16);
    const __nv_bfloat162 a = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&p01), s2);
    const __nv_bfloat162 c = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&p23), s2);
    out[2 * h] = *reinterpret_cast<const uint32_t*>(&a);
    out[2 * h + 1] = *reinterpret_cast<const uint32_t*>(&c);
  }
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
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

__global__ void __launch_bounds__(THREADS, 1) mla_tc_kernel(const __grid_constant__ CUtensorMap tmQ, MlaParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();  // queries, top-k lists, sequence lengths and the cache come from earlier kernels
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* qfull = reinterpret_cast<uint64_t*>(smem + Smem::BAR);  // Q slabs in shared memory landed
  uint64_t* qtm = qfull + 1;                                          // Q slabs in TMEM written
  uint64_t* kfull = qtm + 1;
  uint64_t* kempty = kfull + STAGES;
  uint64_t* sfull = kempty + STAGES;
  uint64_t* pfull = sfull + 2;
  uint64_t* odone = pfull + 2;  // the last PV MMA is complete
  uint64_t* drain = odone + 1;  // every MMA of this CTA is complete
  uint64_t* pvbar = drain + 1;  // one completion per PV MMA group
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Smem::MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile uint32_t* valid = reinterpret_cast<volatile uint32_t*>(smem + Smem::VALID);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Unit: token t, heads [h0, h0 + 128), value half vh, key split.
  const int t = blockIdx.x;
  const int h0 = (blockIdx.y >> 1) * ROWS, vh = blockIdx.y & 1, split = blockIdx.z;
  const int b = request_of(p.q_start, p.B, t);
  const int64_t qs = p.q_start[b], ql = p.q_start[b + 1] - qs, seq = p.seq_lens[b];
  const int64_t qpos = seq - ql + (t - qs);
  const int64_t nkeys = p.topk ? static_cast<int64_t>(p.topk_k) : qpos + 1;
  const int tiles_all = static_cast<int>((nkeys + KT - 1) / KT);
  const int per = (tiles_all + p.nsplit - 1) / p.nsplit;
  const int tg0 = min(split * per, tiles_all), tg1 = min(tg0 + per, tiles_all);
  const int n = tg1 - tg0;  // key tiles of this unit
  const bool fp4 = p.latent_fp4 != nullptr;  // NVFP4 latent rows, decoded by the producers

  if (threadIdx.x == 0) {
    mbar_init(qfull, 1);
    mbar_init(qtm, 4);  // the four softmax warps
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kfull[s], PROD_WARPS * 32);  // every producer lane, once its copies landed
      mbar_init(&kempty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&pfull[i], 4);  // the four softmax warps
    }
    mbar_init(odone, 1);
    mbar_init(drain, 1);
    mbar_init(pvbar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmQ)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(T_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  // Optional cycle counters (p.stamps, [grid][8]): [0] producer waiting for a free stage  [1] producer
  // issuing a tile's copies  [2] MMA waiting for keys  [3] MMA waiting for P  [4] softmax waiting for S
  // [5] rescales  [6] CTA cycles  [7] tiles
  unsigned long long cyc[6] = {0, 0, 0, 0, 0, 0};
  const unsigned long long cta_c0 = clock64();
  auto raise = [&](int code) {
    if (p.err) atomicCAS(p.err, 0, code);
    *abort_flag = 1;
  };
  const int pw = warp == 0 ? 0 : warp - 5;  // producer index of warps 0, 6-12

  if (warp == 0 || warp >= 6) {
    // ------------------------------------------------------------------ producers
    if (warp == 0 && lane == 0 && n > 0) {
      mbar_expect_tx(qfull, QS * Q_SLAB);
      for (int s = 0; s < QS; ++s) tma_load_2d(smem + Smem::Q + s * Q_SLAB, &tmQ, s * 64, t * p.H + h0, qfull);
    }
    const int32_t* bt = p.block_tables + static_cast<int64_t>(b) * p.bt_stride;
    const char* lat = reinterpret_cast<const char*>(p.latent);
    // This lane's key of tile jj: its top-k position (-1: none) and its cache row (row 0 for a masked key,
    // whose scores are dropped).  The two dependent loads run ahead of the tile that uses them: tile j + 2's
    // position and tile j + 1's row are fetched while tile j is processed.
    auto pos_of = [&](int jj) -> int64_t {
      const int64_t kp = static_cast<int64_t>(tg0 + jj) * KT + lane;
      if (jj >= n || kp >= nkeys) return -1;
      return p.topk ? static_cast<int64_t>(p.topk[static_cast<int64_t>(t) * p.topk_k + kp]) : kp;
    };
    auto row_of = [&](int64_t pos) -> int64_t {
      return (pos >= 0 && pos <= qpos) ? static_cast<int64_t>(bt[pos >> 6]) * 64 + (pos & 63) : 0;
    };
    int64_t pos_c = pos_of(0), row_c = row_of(pos_c), pos_n = pos_of(1), row_n = 0, pos_nn = -1;
    // NVFP4: 8 lanes per key, lane q8 with one 64-dim slab of the packed row (4 blocks of 16 values); a
    // tile's packed bytes are loaded before its free-stage wait.
    const int fr = 4 * pw + (lane >> 3), q8 = lane & 7;
    for (int j = 0; j < n; ++j) {
      const int st = j % STAGES;
      const unsigned long long c0 = clock64();
      if (j > 0) {
        pos_c = pos_n;
        row_c = row_n;
        pos_n = pos_nn;
      }
      const bool ok = pos_c >= 0 && pos_c <= qpos;
      const int64_t row = row_c;
      const uint32_t mask = __ballot_sync(0xffffffffu, ok);
      row_n = row_of(pos_n);   // used by the next tile
      pos_nn = pos_of(j + 2);  // used two tiles from now
      uint4 w0, w1;
      uint32_t scw = 0, ro[4];
      if (fp4) {
        const uint8_t* fsrc = p.latent_fp4 + __shfl_sync(0xffffffffu, row, fr) * kFp4Row;
        const uint4* pk = reinterpret_cast<const uint4*>(fsrc + q8 * 32);
        w0 = __ldg(pk);
        w1 = __ldg(pk + 1);
        const uint2 rw = __ldg(reinterpret_cast<const uint2*>(fsrc + kFp4Rope + q8 * 8));
        const uint32_t sw = __ldg(reinterpret_cast<const uint32_t*>(fsrc + kFp4Scales + q8 * 4));  // scale word q8
        // Before the free-stage wait: block 4 q8 + blk's scale sits at byte 8 blk + q8 of the scale region
        // (word 2 blk + q8 / 4, loaded by that lane of the key's eight; byte q8 % 4), and rope chunk q8 is
        // converted to bf16.
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
          const uint32_t wd = __shfl_sync(0xffffffffu, sw, (lane & ~7) | (2 * blk + (q8 >> 2)));
          scw |= ((wd >> (8 * (q8 & 3))) & 0xFFu) << (8 * blk);
        }
        e4m3x8_to_bf16(rw, ro);
      }
      if (j >= STAGES && !__all_sync(0xffffffffu, mbar_wait(&kempty[st], ((j / STAGES) - 1) & 1, abort_flag))) {
        if (lane == 0) raise(501);
        break;
      }
      const unsigned long long c1 = clock64();
      cyc[0] += c1 - c0;
      if (warp == 0 && lane == 0) valid[st] = mask;  // published by the barrier's completion
      uint8_t* kdst = smem + Smem::K + st * K_BYTES;
      if (fp4) {
        // Decode slab q8 into bf16 chunks of the swizzled tile and store rope chunk q8.  A code times its block
        // scale has at most 5 significant bits and an e4m3 value 4, so the bf16 values are exact.
        const int r = fr;
        uint8_t* krow = kdst + r * 128;
        *reinterpret_cast<uint4*>(krow + 8 * K_SLAB + ((q8 ^ (r & 7)) << 4)) = make_uint4(ro[0], ro[1], ro[2], ro[3]);
        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint8_t* kslab = krow + q8 * K_SLAB;
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {  // block of latent dims [64 q8 + 16 blk, + 16)
          __nv_fp8_e4m3 f8;
          f8.__x = static_cast<__nv_fp8_storage_t>((scw >> (8 * blk)) & 0xFFu);
          const __nv_bfloat162 sc2 = __float2bfloat162_rn(static_cast<float>(f8));  // exact: 4 significant bits
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // two 16-byte chunks of 8 values
            uint32_t o[4];
            e2m1x8_to_bf16(words[2 * blk + h], sc2, o);
            const int c = blk * 2 + h;
            *reinterpret_cast<uint4*>(kslab + ((c ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
        // the decoded chunks (generic stores) must be visible to the tensor cores
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(&kfull[st]);
        cyc[1] += clock64() - c1;
        continue;
      }
      // Copy `it` moves 4 keys x one 128-byte slab row: 8 lanes per key, one 16-byte chunk each.
#pragma unroll 2
      for (int k = 0; k < COPIES_PER_WARP; ++k) {
        const int it = pw * COPIES_PER_WARP + k;
        const int slab = it >> 3, r = 4 * (it & 7) + (lane >> 3), c = lane & 7;
        const int64_t rr = __shfl_sync(0xffffffffu, row, r);
        const uint32_t dst = smem_addr(kdst + slab * K_SLAB + r * 128 + ((c ^ (r & 7)) << 4));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst),
                     "l"(lat + rr * (C * 2) + slab * 128 + c * 16)
                     : "memory");
      }
      // fires once this lane's copies have landed; the barrier expects every producer lane
      asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(&kfull[st])) : "memory");
      cyc[1] += clock64() - c1;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && n > 0) {
      constexpr uint32_t IS = idesc_bf16(ROWS, KT, false);  // S = Q K^T: both K-major
      constexpr uint32_t IP = idesc_bf16(ROWS, VH, true);   // O += P V: V MN-major
      const uint32_t kbase = smem_addr(smem + Smem::K);
      const uint64_t qd = sw128_desc(smem_addr(smem + Smem::Q));
      bool ok = mbar_wait(qfull, 0, abort_flag) && mbar_wait(qtm, 0, abort_flag);
      if (!ok) raise(502);
      fence_after();
      for (int j = 0; ok && j <= n; ++j) {
        if (j < n) {  // S_j
          const int st = j % STAGES;
          const unsigned long long c0 = clock64();
          if (!mbar_wait(&kfull[st], (j / STAGES) & 1, abort_flag)) {
            raise(503);
            break;
          }
          cyc[2] += clock64() - c0;
          fence_after();
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // cp.async data -> tensor cores
          // Descriptors advance by adding the byte offset / 16 to their start-address field (shared memory
          // addresses stay below 2^18, so the 14-bit field never carries), and both loops unroll fully: the
          // single issuing thread spends a few instructions per MMA instead of rebuilding descriptors.
          const uint32_t d = tmem + T_S + (j & 1) * KT;
          const uint64_t kd = sw128_desc(kbase + st * K_BYTES);
#pragma unroll
          for (int s = 0; s < QS; ++s)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16(d, qd + static_cast<uint64_t>((s * Q_SLAB + kk * 32) >> 4),
                       kd + static_cast<uint64_t>((s * K_SLAB + kk * 32) >> 4), IS, (s | kk) ? 1u : 0u);
#pragma unroll
          for (int s = QS; s < SLABS; ++s)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)  // Q from TMEM: 16 dims = 8 columns per MMA
              mma_bf16_ts(d, tmem + T_Q + (s - QS) * 32 + kk * 8, kd + static_cast<uint64_t>((s * K_SLAB + kk * 32) >> 4),
                          IS, 1u);
          mma_commit(&sfull[j & 1]);
        }
        if (j >= 1) {  // O += P_{j-1} V_{j-1}
          const int i = j - 1, st = i % STAGES;
          const unsigned long long c0 = clock64();
          if (!mbar_wait(&pfull[i & 1], (i >> 1) & 1, abort_flag)) {
            raise(504);
            break;
          }
          cyc[3] += clock64() - c0;
          fence_after();
          // this half's 4 slabs of 64 value columns; 16 keys per MMA: 16 rows of 128 B, two 8-row atoms
          const uint64_t vd = sw128_mn_desc(kbase + st * K_BYTES + vh * 4 * K_SLAB, K_SLAB, 1024);
#pragma unroll
          for (int kk = 0; kk < 2; ++kk)
            mma_bf16_ts(tmem + T_O, tmem + T_P + (i & 1) * 16 + kk * 8, vd + static_cast<uint64_t>((kk * 2048) >> 4), IP,
                        (i > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&kempty[st]);
          mma_commit(pvbar);
          if (i == n - 1) mma_commit(odone);
        }
      }
      mma_commit(drain);
      (void)mbar_wait_drain(drain, 0);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const uint32_t tl = static_cast<uint32_t>(quarter * 32) << 16;
    if (n > 0) {  // Q slabs QS.. of this thread's head row -> TMEM (bf16 pairs, 32 columns per slab)
      const uint4* qrow = reinterpret_cast<const uint4*>(p.q + (static_cast<int64_t>(t) * p.H + h0 + row) * C);
#pragma unroll 1
      for (int s = QS; s < SLABS; ++s) {
        uint32_t w[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 v = qrow[s * 8 + i];
          w[4 * i] = v.x;
          w[4 * i + 1] = v.y;
          w[4 * i + 2] = v.z;
          w[4 * i + 3] = v.w;
        }
        tmem_st32(tmem + tl + T_Q + (s - QS) * 32, reinterpret_cast<const float*>(w));
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(qtm);
    }
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int bs = j & 1;
      const unsigned long long c0 = clock64();
      // kfull_j (complete once S_j is) publishes the tile's key-validity mask
      if (!__all_sync(0xffffffffu, mbar_wait(&sfull[bs], (j >> 1) & 1, abort_flag) &&
                                       mbar_wait(&kfull[j % STAGES], (j / STAGES) & 1, abort_flag))) {
        if (lane == 0) raise(505);
        ok = false;
        break;
      }
      cyc[4] += clock64() - c0;
      fence_after();
      const uint32_t vmask = valid[j % STAGES];
      float s[32];
      tmem_ld32(tmem + tl + T_S + bs * KT, s);
      float mx = -INFINITY;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        s[k] = ((vmask >> k) & 1u) ? s[k] * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, s[k]);
      }
      // The running maximum is only raised when it grows by more than 8 (2^8 in the exp2 domain); a row
      // that had no valid key yet holds O = 0 and needs no rescale.
      const bool grow = mx > m_used + 8.f;
      const bool rescale = grow && m_used != -INFINITY;
      if (__any_sync(0xffffffffu, rescale)) {
        // O must hold P_{j-1} V_{j-1}: wait for the j-th PV completion (sfull_j already implies the
        // (j-1)-th, and PV_j cannot start before this tile's P is published, so the parity is unambiguous)
        if (!__all_sync(0xffffffffu, mbar_wait(pvbar, (j - 1) & 1, abort_flag))) {
          if (lane == 0) raise(506);
          ok = false;
          break;
        }
        fence_after();
        cyc[5] += 1;
        const float alpha = rescale ? exp2f(m_used - mx) : 1.f;
#pragma unroll 1
        for (int c = 0; c < VH; c += 32) {
          float o[32];
          tmem_ld32(tmem + tl + T_O + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(tmem + tl + T_O + c, o);
        }
        l *= alpha;
      }
      if (grow) m_used = mx;
      const float base = m_used == -INFINITY ? 0.f : m_used;
      uint32_t pk[16];
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float p0 = exp2f(s[2 * i] - base), p1 = exp2f(s[2 * i + 1] - base);
        sum += p0 + p1;
        pk[i] = pack_bf16(p0, p1);
      }
      l += sum;
      tmem_st16(tmem + tl + T_P + bs * 16, pk);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[bs]);
    }
    if (ok && n > 0 && !__all_sync(0xffffffffu, mbar_wait(odone, 0, abort_flag))) {
      if (lane == 0) raise(507);
      ok = false;
    }
    if (ok) {
      fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int64_t th = static_cast<int64_t>(t) * p.H + h0 + row;
      const int64_t prow = th * p.nsplit + split;
#pragma unroll 1
      for (int c = 0; c < VH; c += 32) {
        float o[32];
        if (n > 0) {
          tmem_ld32(tmem + tl + T_O + c, o);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (p.nsplit == 1) {
          uint4* dst = reinterpret_cast<uint4*>(p.out + th * (2 * VH) + vh * VH + c);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            dst[q4] = make_uint4(pack_bf16(o[8 * q4] * inv, o[8 * q4 + 1] * inv),
                                 pack_bf16(o[8 * q4 + 2] * inv, o[8 * q4 + 3] * inv),
                                 pack_bf16(o[8 * q4 + 4] * inv, o[8 * q4 + 5] * inv),
                                 pack_bf16(o[8 * q4 + 6] * inv, o[8 * q4 + 7] * inv));
        } else {
          float4* dst = reinterpret_cast<float4*>(p.part_o + prow * (2 * VH) + vh * VH + c);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4)
            dst[q4] = make_float4(o[4 * q4] * inv, o[4 * q4 + 1] * inv, o[4 * q4 + 2] * inv, o[4 * q4 + 3] * inv);
        }
      }
      if (p.nsplit > 1 && vh == 0) {
        p.part_ml[prow * 2] = m_used;
        p.part_ml[prow * 2 + 1] = l;
      }
    }
  }
  if (p.stamps && lane == 0) {
    unsigned long long* st = p.stamps + ((static_cast<int64_t>(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x +
                                         blockIdx.x) * 8;
    if (warp == 0) {
      st[0] = cyc[0];
      st[1] = cyc[1];
      st[7] = n;
    }
    if (warp == 1) {
      st[2] = cyc[2];
      st[3] = cyc[3];
    }
    if (warp == 2) {
      st[4] = cyc[4];
      st[5] = cyc[5];
      st[6] = clock64() - cta_c0;
    }
  }
  if ((warp == 0 || warp >= 6) && *abort_flag) {
    // copies issued before the abort complete within microseconds: wait for this lane's
    asm volatile("cp.async.wait_all;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(T_COLS));
  }
}

}  // namespace mlatc
}  // namespace shk

namespace {

using namespace shk::mlatc;

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

// bf16 [rows][576] (row stride 1152 B), box {64 columns, box_rows}, 128-byte swizzle.
int encode_rows(CUtensorMap* m, const void* base, int64_t rows, int box_rows) {
  auto enc = encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(C) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

constexpr int kMaxDevices = 64;

}  // namespace

extern "C" int sh_mla_decode_tc(const MlaParams* p, cudaStream_t stream) {
  if ((!p->latent && !p->latent_fp4) || p->H % ROWS != 0) return -2;
  if (p->T <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(p->q) & 15) || (reinterpret_cast<uintptr_t>(p->latent) & 15) ||
      (reinterpret_cast<uintptr_t>(p->latent_fp4) & 15))
    return -2;
  CUtensorMap mq;
  const int r = encode_rows(&mq, p->q, static_cast<int64_t>(p->T) * p->H, ROWS);
  if (r) return 1000 + r;
  static bool ready[kMaxDevices] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = 0;
  if (!ready[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(mla_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::TOTAL);
    if (e != cudaSuccess) return static_cast<int>(e);
    ready[dev] = true;
  }
  shk::launch(mla_tc_kernel, dim3(p->T, (p->H / ROWS) * 2, p->nsplit), dim3(THREADS), Smem::TOTAL, stream, mq, *p);
  return static_cast<int>(cudaGetLastError());
}
