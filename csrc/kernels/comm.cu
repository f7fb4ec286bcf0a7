// Tensor-parallel all-reduce over NVLink peer memory, fused with the next
// layer's residual add + RMSNorm.
//
// The row-parallel GEMM writes its [T, H] partial into local memory; this
// kernel moves data only with P2P STORES (posted writes, no round trip):
//   one-shot (small T*H): every rank pushes its partial rows into a receive
//     slot of every peer, waits for the peers' pushes, and sums the world
//     partials in rank order from its own memory;
//   two-shot (large T*H): rows are split into world contiguous chunks; every
//     rank pushes each chunk to its owner, the owner sums its chunk in rank
//     order and pushes the bf16 sums into every rank's gather buffer, and each
//     rank reads the gathered sums from its own memory;
// then residual += sum, out = rms_norm(residual) * weight (or out = sum) on
// every rank.  The summation order is the same everywhere, so all ranks hold
// bit-identical results.
//
// Synchronisation: block b of every rank handles the same rows, so ranks only
// synchronise block-to-block: a system-scope release store of the block's
// epoch into each peer's flag slot, then acquire loads of the peers' slots.
// Receive and gather buffers are double-buffered by epoch parity, which makes
// a trailing "peers are done reading" barrier unnecessary: before a rank can
// write a slot of parity e again (call e + 2) it must pass call e + 1's wait,
// which every peer signals only after finishing call e.  The grid is the same
// for every call of a communicator, so all blocks of a call share one epoch
// (and one parity), and at most one block per SM so every block is resident
// while it waits.  Each wait gives up after a time limit, records an error
// code in *err and skips the remaining data phases (no trap, no hang).
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "comm.h"
#include "pdl.cuh"

namespace shk {
namespace comm {

constexpr uint64_t kTimeoutNs = 5000000000ull;  // 5 s

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t* flag_slot(uint32_t* pad, int phase, int block, int src) {
  return pad + (static_cast<size_t>(phase) * SH_COMM_MAX_BLOCKS + block) * SH_COMM_MAX_WORLD + src;
  static_assert(SH_COMM_PHASES == 3, "flag layout");
}

// Cross-rank barrier between same-index blocks. Returns false on timeout.
__device__ bool barrier_flags(uint32_t* const* peer_flags, int world, int rank, int* err, int phase, uint32_t epoch,
                              volatile int* bail, unsigned long long wait_ns) {
  const uint64_t limit = wait_ns ? wait_ns : kTimeoutNs;
  __syncthreads();
  if (threadIdx.x < world) {
    // st.release orders every store the block made before the bar.sync above
    // (cumulativity) ahead of the flag, at system scope.
    st_release(flag_slot(peer_flags[threadIdx.x], phase, blockIdx.x, rank), epoch);
  }
  if (threadIdx.x < world) {
    const uint32_t* f = flag_slot(peer_flags[rank], phase, blockIdx.x, threadIdx.x);
    const uint64_t t0 = now_ns();
    while (static_cast<int32_t>(ld_acquire(f) - epoch) < 0) {
      if (*bail || now_ns() - t0 > limit) {
        *bail = 1;
        if (err) atomicCAS(err, 0, 100 + phase);
        break;
      }
    }
  }
  __syncthreads();
  return *bail == 0;
}

__device__ __forceinline__ bool barrier(const ArParams& p, int phase, uint32_t epoch, volatile int* bail) {
  return barrier_flags(p.peer_flags, p.world, p.rank, p.err, phase, epoch, bail, p.wait_ns);
}

__device__ __forceinline__ void add8(float* acc, uint4 v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float* v) {
  uint4 r;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  return r;
}

// L2 prefetch of block b's slice of [base, base + bytes): the weights of the
// GEMM that follows the collective are static, so the fetch is issued before
// griddepcontrol.wait and proceeds while the ranks push and wait.
__device__ __forceinline__ void l2_prefetch_slice(const void* base, unsigned long long bytes) {
  if (base == nullptr || bytes < 16 || threadIdx.x != 0) return;
  const unsigned long long per = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
  const unsigned long long lo = static_cast<unsigned long long>(blockIdx.x) * per;
  const unsigned long long hi = lo + per < bytes ? lo + per : bytes;
  for (unsigned long long off = lo; off + 16 <= hi; off += (1u << 20)) {
    const unsigned long long left = hi - off;
    const uint32_t n = static_cast<uint32_t>(left < (1u << 20) ? left : (1u << 20)) & ~15u;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(static_cast<const char*>(base) + off), "r"(n)
                 : "memory");
  }
}

// Rows are processed by groups of kGroupThreads threads (four warps); a block
// runs blockDim.x / kGroupThreads groups on different rows at once, so decode
// sizes (tens to hundreds of rows) are handled in one pass instead of one row
// per block at a time.  Thread t of a group owns the 8-element vectors
// v = t + k * kGroupThreads (k < VPT) of its row.
constexpr int kGroupThreads = 128;

// Sum over the threads of this thread's group (shuffles + one named barrier per group).
__device__ __forceinline__ float group_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int g = threadIdx.x / kGroupThreads, w = (threadIdx.x % kGroupThreads) >> 5;
  if ((threadIdx.x & 31) == 0) red[g * 4 + w] = v;
  asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(kGroupThreads) : "memory");
  const float t = red[g * 4] + red[g * 4 + 1] + red[g * 4 + 2] + red[g * 4 + 3];
  asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(kGroupThreads) : "memory");
  return t;
}

// residual += sum (bf16), out = rms_norm(residual) * w for one row (or out = sum).
template <int VPT>
__device__ void finish_row(const ArParams& p, int64_t r, float (*acc)[8], float* red) {
  const int nv = p.H / 8;
  const int lt = threadIdx.x % kGroupThreads;
  if (!p.fuse_norm) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = lt + k * kGroupThreads;
      if (v < nv) reinterpret_cast<uint4*>(p.out + r * p.H)[v] = pack8(acc[k]);
    }
    return;
  }
  float ss = 0.f;
  uint4 res[VPT];
  uint4 rv[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = lt + k * kGroupThreads;
    if (v < nv) rv[k] = reinterpret_cast<const uint4*>(p.residual + r * p.H)[v];
  }
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = lt + k * kGroupThreads;
    if (v >= nv) continue;
    float sum[8];
    const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&rv[k]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(rh[i]);
      sum[2 * i] = f.x + acc[k][2 * i];
      sum[2 * i + 1] = f.y + acc[k][2 * i + 1];
    }
    res[k] = pack8(sum);  // the residual stream is stored in bf16
    const __nv_bfloat162* q = reinterpret_cast<const __nv_bfloat162*>(&res[k]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(q[i]);
      ss += f.x * f.x + f.y * f.y;
    }
    reinterpret_cast<uint4*>(p.residual + r * p.H)[v] = res[k];
  }
  const float inv = rsqrtf(group_sum(ss, red) / p.H + p.eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = lt + k * kGroupThreads;
    if (v >= nv) continue;
    const uint4 wv = reinterpret_cast<const uint4*>(p.weight)[v];
    const __nv_bfloat162* q = reinterpret_cast<const __nv_bfloat162*>(&res[k]);
    const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wv);
    float o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(q[i]);
      const float2 g = __bfloat1622float2(wh[i]);
      o[2 * i] = f.x * inv * g.x;
      o[2 * i + 1] = f.y * inv * g.y;
    }
    reinterpret_cast<uint4*>(p.out + r * p.H)[v] = pack8(o);
  }
}

template <int VPT>
__device__ __forceinline__ void zero_acc(float (*acc)[8]) {
#pragma unroll
  for (int k = 0; k < VPT; ++k)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[k][i] = 0.f;
}

// acc += the row's vectors (all loads of the row issued before any use).
template <int VPT>
__device__ __forceinline__ void add_row(float (*acc)[8], const uint4* src, int nv) {
  const int lt = threadIdx.x % kGroupThreads;
  uint4 val[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = lt + k * kGroupThreads;
    val[k] = v < nv ? src[v] : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int k = 0; k < VPT; ++k) add8(acc[k], val[k]);
}

// dst[d][v] = src[v] for this thread's vectors of one row.
template <int VPT>
__device__ __forceinline__ void push_row(const uint4* src, uint4* const* dst, int ndst, int nv) {
  const int lt = threadIdx.x % kGroupThreads;
  uint4 val[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = lt + k * kGroupThreads;
    if (v < nv) val[k] = src[v];
  }
  for (int d = 0; d < ndst; ++d)
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = lt + k * kGroupThreads;
      if (v < nv) dst[d][v] = val[k];
    }
}

// ---- compressed rows (ArParams::quant): [H codes | H / 128 fp32 scales] in a bf16 row slot ----------
// A block of 128 elements is 16 consecutive 8-element vectors, i.e. one half-warp of a row group (thread t
// of a group owns vectors t + k * 128), so a block's amax is a 4-step shuffle reduction.
constexpr int kQBlock = 128;

__device__ __forceinline__ float half_warp_max(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// 8 values -> 8 codes (int8: round(x / s) in [-127, 127]; fp8: e4m3(x / s)) with s = amax / qmax.
__device__ __forceinline__ uint2 encode8(const float* x, float amax, int quant, float* scale) {
  const float qmax = quant == 1 ? 127.f : 448.f;
  *scale = amax / qmax;
  const float inv = amax > 0.f ? qmax / amax : 0.f;
  uint32_t w[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t c;
    if (quant == 1) {
      const float q = fminf(fmaxf(rintf(x[i] * inv), -127.f), 127.f);
      c = static_cast<uint32_t>(static_cast<int32_t>(q)) & 0xFFu;
    } else {
      __nv_fp8_e4m3 f(fminf(fmaxf(x[i] * inv, -448.f), 448.f));
      c = f.__x;
    }
    w[i >> 2] |= c << (8 * (i & 3));
  }
  return make_uint2(w[0], w[1]);
}
__device__ __forceinline__ void decode8_add(float* acc, uint2 code, float scale, int quant) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t c = ((i < 4 ? code.x : code.y) >> (8 * (i & 3))) & 0xFFu;
    float v;
    if (quant == 1) {
      v = static_cast<float>(static_cast<int8_t>(c));
    } else {
      __nv_fp8_e4m3 f;
      f.__x = static_cast<__nv_fp8_storage_t>(c);
      v = static_cast<float>(f);
    }
    acc[i] += v * scale;
  }
}
// Encode this thread's vectors of one row (fp32 values in x) and store codes + block scales into every dst.
template <int VPT>
__device__ __forceinline__ void push_row_q(float (*x)[8], char* const* dst, int ndst, int nv, int quant) {
  const int lt = threadIdx.x % kGroupThreads;
  const bool lead = (threadIdx.x & 15) == 0;
  uint2 code[VPT];
  float scale[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(x[k][i]));
    code[k] = encode8(x[k], half_warp_max(am), quant, &scale[k]);
  }
  const size_t H = static_cast<size_t>(nv) * 8;
  for (int d = 0; d < ndst; ++d)
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = lt + k * kGroupThreads;
      if (v >= nv) continue;
      reinterpret_cast<uint2*>(dst[d])[v] = code[k];
      if (lead) reinterpret_cast<float*>(dst[d] + H)[v >> 4] = scale[k];
    }
}
// acc += the dequantised row (all loads issued before any use).
template <int VPT>
__device__ __forceinline__ void add_row_q(float (*acc)[8], const char* src, int nv, int quant) {
  const int lt = threadIdx.x % kGroupThreads;
  const size_t H = static_cast<size_t>(nv) * 8;
  uint2 code[VPT];
  float scale[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = lt + k * kGroupThreads;
    code[k] = v < nv ? reinterpret_cast<const uint2*>(src)[v] : make_uint2(0u, 0u);
    scale[k] = v < nv ? reinterpret_cast<const float*>(src + H)[v >> 4] : 0.f;
  }
#pragma unroll
  for (int k = 0; k < VPT; ++k) decode8_add(acc[k], code[k], scale[k], quant);
}
// This thread's vectors of a bf16 row as fp32 (zero past the row end).
template <int VPT>
__device__ __forceinline__ void load_row_f32(float (*x)[8], const uint4* src, int nv) {
  zero_acc<VPT>(x);
  add_row<VPT>(x, src, nv);
}

template <int VPT, bool QUANT>
__global__ void __launch_bounds__(512) allreduce_kernel(ArParams p) {
  shk::pdl_trigger();
  l2_prefetch_slice(p.prefetch, p.prefetch_bytes);
  shk::pdl_wait();
  __shared__ float red[32];
  __shared__ uint32_t s_epoch;
  __shared__ volatile int bail;
  if (threadIdx.x == 0) {
    s_epoch = ++p.counters[blockIdx.x];
    bail = 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const size_t par = epoch & 1u;
  unsigned long long* stamp =
      (p.timing && blockIdx.x == 0 && threadIdx.x == 0) ? p.timing + 4 * (epoch % 64u) : nullptr;
  if (stamp) stamp[0] = now_ns();
  const int nv = p.H / 8;
  const int G = blockDim.x / kGroupThreads;            // row groups per block
  const int g = threadIdx.x / kGroupThreads;
  const int64_t slots = static_cast<int64_t>(gridDim.x) * G;  // rows in flight per pass
  const int64_t slot0 = static_cast<int64_t>(blockIdx.x) * G + g;
  const int W = p.world;
  const size_t H = static_cast<size_t>(p.H);
  auto recv_row = [&](int dst, int src, int64_t r) {
    return reinterpret_cast<uint4*>(p.peer_recv[dst] + ((par * W + src) * p.max_T + r) * H);
  };
  auto gather_row = [&](int dst, int64_t r) {
    return reinterpret_cast<uint4*>(p.peer_gather[dst] + (par * p.max_T + r) * H);
  };
  const uint4* partial = reinterpret_cast<const uint4*>(p.partial);
  uint4* dsts[SH_COMM_MAX_WORLD];

  if constexpr (QUANT) {
    // Compressed rows.  Every contribution is encoded once and written to its readers' slots, its own
    // rank's included, so all ranks decode the same bytes.
    auto qrecv = [&](int dst, int src, int64_t r) { return reinterpret_cast<char*>(recv_row(dst, src, r)); };
    auto qgather = [&](int dst, int64_t r) { return reinterpret_cast<char*>(gather_row(dst, r)); };
    char* qd[SH_COMM_MAX_WORLD];
    if (!p.two_shot) {
      for (int64_t r = slot0; r < p.T; r += slots) {
        float x[VPT][8];
        load_row_f32<VPT>(x, partial + r * (H / 8), nv);
        for (int d = 0; d < W; ++d) qd[d] = qrecv(d, p.rank, r);
        push_row_q<VPT>(x, qd, W, nv, p.quant);
      }
      if (stamp) stamp[1] = now_ns();
      if (!barrier(p, 0, epoch, &bail)) return;
      if (stamp) stamp[2] = now_ns();
      for (int64_t r = slot0; r < p.T; r += slots) {
        float acc[VPT][8];
        zero_acc<VPT>(acc);
        for (int src = 0; src < W; ++src) add_row_q<VPT>(acc, qrecv(p.rank, src, r), nv, p.quant);
        finish_row<VPT>(p, r, acc, red);
      }
      if (stamp) stamp[3] = now_ns();
      return;
    }
    const int Tc = (p.T + W - 1) / W;
    for (int i = 0; i < W; ++i) {  // chunk rows to their owners (this rank's own chunk included)
      const int o = (p.rank + i) % W;
      const int64_t r1 = min(static_cast<int64_t>(p.T), static_cast<int64_t>(o + 1) * Tc);
      for (int64_t r = static_cast<int64_t>(o) * Tc + slot0; r < r1; r += slots) {
        float x[VPT][8];
        load_row_f32<VPT>(x, partial + r * (H / 8), nv);
        qd[0] = qrecv(o, p.rank, r);
        push_row_q<VPT>(x, qd, 1, nv, p.quant);
      }
    }
    if (stamp) stamp[1] = now_ns();
    if (!barrier(p, 0, epoch, &bail)) return;
    if (stamp) stamp[2] = now_ns();
    {  // owner: decode and sum in rank order, requantise the sum into every rank's gather slot
      const int64_t r1 = min(static_cast<int64_t>(p.T), static_cast<int64_t>(p.rank + 1) * Tc);
      for (int64_t r = static_cast<int64_t>(p.rank) * Tc + slot0; r < r1; r += slots) {
        float acc[VPT][8];
        zero_acc<VPT>(acc);
        for (int src = 0; src < W; ++src) add_row_q<VPT>(acc, qrecv(p.rank, src, r), nv, p.quant);
        for (int d = 0; d < W; ++d) qd[d] = qgather(d, r);
        push_row_q<VPT>(acc, qd, W, nv, p.quant);
      }
    }
    if (!barrier(p, 1, epoch, &bail)) return;
    for (int o = 0; o < W; ++o) {
      const int64_t r1 = min(static_cast<int64_t>(p.T), static_cast<int64_t>(o + 1) * Tc);
      for (int64_t r = static_cast<int64_t>(o) * Tc + slot0; r < r1; r += slots) {
        float acc[VPT][8];
        zero_acc<VPT>(acc);
        add_row_q<VPT>(acc, qgather(p.rank, r), nv, p.quant);
        finish_row<VPT>(p, r, acc, red);
      }
    }
    if (stamp) stamp[3] = now_ns();
    return;
  }

  if (!p.two_shot) {
    for (int64_t r = slot0; r < p.T; r += slots) {
      int n = 0;
      for (int i = 1; i < W; ++i) dsts[n++] = recv_row((p.rank + i) % W, p.rank, r);
      push_row<VPT>(partial + r * (H / 8), dsts, n, nv);
    }
    if (stamp) stamp[1] = now_ns();
    if (!barrier(p, 0, epoch, &bail)) return;  // every peer's partial has landed here
    if (stamp) stamp[2] = now_ns();
    for (int64_t r = slot0; r < p.T; r += slots) {
      float acc[VPT][8];
      zero_acc<VPT>(acc);
      for (int src = 0; src < W; ++src)
        add_row<VPT>(acc, src == p.rank ? partial + r * (H / 8) : recv_row(p.rank, src, r), nv);
      finish_row<VPT>(p, r, acc, red);
    }
    if (stamp) stamp[3] = now_ns();
    return;
  }
  // Two-shot.  Owner o holds rows [o*Tc, min(T, (o+1)*Tc)); slot s of every
  // rank handles local row indices j = s, s + slots, ... of every chunk.
  const int Tc = (p.T + W - 1) / W;
  for (int i = 1; i < W; ++i) {
    const int o = (p.rank + i) % W;
    const int64_t r1 = min(static_cast<int64_t>(p.T), static_cast<int64_t>(o + 1) * Tc);
    for (int64_t r = static_cast<int64_t>(o) * Tc + slot0; r < r1; r += slots) {
      dsts[0] = recv_row(o, p.rank, r);
      push_row<VPT>(partial + r * (H / 8), dsts, 1, nv);
    }
  }
  if (stamp) stamp[1] = now_ns();
  if (!barrier(p, 0, epoch, &bail)) return;  // every chunk this rank owns has landed
  if (stamp) stamp[2] = now_ns();
  {
    const int64_t r1 = min(static_cast<int64_t>(p.T), static_cast<int64_t>(p.rank + 1) * Tc);
    for (int64_t r = static_cast<int64_t>(p.rank) * Tc + slot0; r < r1; r += slots) {
      float acc[VPT][8];
      zero_acc<VPT>(acc);
      for (int src = 0; src < W; ++src)
        add_row<VPT>(acc, src == p.rank ? partial + r * (H / 8) : recv_row(p.rank, src, r), nv);
      const int lt = threadIdx.x % kGroupThreads;
      uint4 packed[VPT];
#pragma unroll
      for (int k = 0; k < VPT; ++k) packed[k] = pack8(acc[k]);
      for (int i = 0; i < W; ++i) {
        uint4* dst = gather_row((p.rank + i) % W, r);
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
          const int v = lt + k * kGroupThreads;
          if (v < nv) dst[v] = packed[k];
        }
      }
    }
  }
  if (!barrier(p, 1, epoch, &bail)) return;  // every owner's sums have landed here
  for (int o = 0; o < W; ++o) {
    const int64_t r1 = min(static_cast<int64_t>(p.T), static_cast<int64_t>(o + 1) * Tc);
    for (int64_t r = static_cast<int64_t>(o) * Tc + slot0; r < r1; r += slots) {
      float acc[VPT][8];
      zero_acc<VPT>(acc);
      add_row<VPT>(acc, gather_row(p.rank, r), nv);
      finish_row<VPT>(p, r, acc, red);
    }
  }
  if (stamp) stamp[3] = now_ns();
}


template <int VPT>
__global__ void __launch_bounds__(512) rs_norm_ag_kernel(RsParams p) {
  shk::pdl_trigger();
  l2_prefetch_slice(p.prefetch, p.prefetch_bytes);
  shk::pdl_wait();
  __shared__ float red[32];
  __shared__ uint32_t s_epoch, s_target;
  __shared__ volatile int bail;
  if (threadIdx.x == 0) {
    s_epoch = ++p.counters[blockIdx.x];
    const uint32_t par = s_epoch & 1u;
    s_target = p.targets[2 * blockIdx.x + par] + p.expected;
    p.targets[2 * blockIdx.x + par] = s_target;
    bail = 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const size_t par = epoch & 1u;
  unsigned long long* stamp =
      (p.timing && blockIdx.x == 0 && threadIdx.x == 0) ? p.timing + 4 * (epoch % 64u) : nullptr;
  if (stamp) stamp[0] = now_ns();
  if (threadIdx.x == 0) {  // every rank's pushed rows for this rank have landed
    const uint32_t* cnt = p.rs_cnt + par;
    const uint64_t t0 = now_ns();
    while (static_cast<int32_t>(ld_acquire(cnt) - s_target) < 0) {
      if (now_ns() - t0 > (p.wait_ns ? p.wait_ns : kTimeoutNs)) {
        bail = 1;
        if (p.err) atomicCAS(p.err, 0, 200);
        break;
      }
    }
  }
  __syncthreads();
  if (bail) return;
  if (stamp) stamp[1] = now_ns();
  const int nv = p.H / 8;
  const int G = blockDim.x / kGroupThreads;
  const int g = threadIdx.x / kGroupThreads;
  const int lt = threadIdx.x % kGroupThreads;
  const int64_t slots = static_cast<int64_t>(gridDim.x) * G;
  const int64_t slot0 = static_cast<int64_t>(blockIdx.x) * G + g;
  const int W = p.world;
  const size_t H = static_cast<size_t>(p.H);
  const int64_t r1 = min(static_cast<int64_t>(p.T), static_cast<int64_t>(p.rank + 1) * p.Tc);
  for (int64_t r = static_cast<int64_t>(p.rank) * p.Tc + slot0; r < r1; r += slots) {
    float acc[VPT][8];
    zero_acc<VPT>(acc);
    for (int src = 0; src < W; ++src)
      add_row<VPT>(acc, reinterpret_cast<const uint4*>(p.recv + ((par * W + src) * p.max_T + r) * H), nv);
    uint4 rv[VPT], res[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = lt + k * kGroupThreads;
      if (v < nv) rv[k] = reinterpret_cast<const uint4*>(p.residual + r * H)[v];
    }
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = lt + k * kGroupThreads;
      if (v >= nv) continue;
      float sum[8];
      const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&rv[k]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(rh[i]);
        sum[2 * i] = f.x + acc[k][2 * i];
        sum[2 * i + 1] = f.y + acc[k][2 * i + 1];
      }
      res[k] = pack8(sum);
      const __nv_bfloat162* q = reinterpret_cast<const __nv_bfloat162*>(&res[k]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(q[i]);
        ss += f.x * f.x + f.y * f.y;
      }
      reinterpret_cast<uint4*>(p.residual + r * H)[v] = res[k];
    }
    const float inv = rsqrtf(group_sum(ss, red) / p.H + p.eps);
    uint4 y[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = lt + k * kGroupThreads;
      if (v >= nv) continue;
      const uint4 wv = reinterpret_cast<const uint4*>(p.weight)[v];
      const __nv_bfloat162* q = reinterpret_cast<const __nv_bfloat162*>(&res[k]);
      const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wv);
      float o[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(q[i]);
        const float2 w2 = __bfloat1622float2(wh[i]);
        o[2 * i] = f.x * inv * w2.x;
        o[2 * i + 1] = f.y * inv * w2.y;
      }
      y[k] = pack8(o);
    }
    for (int i = 0; i < W; ++i) {
      const int d = (p.rank + i) % W;
      uint4* dy = reinterpret_cast<uint4*>(p.peer_gather[d] + (par * p.max_T + r) * H);
      uint4* dr = p.gather_res ? reinterpret_cast<uint4*>(p.peer_gather_res[d] + (par * p.max_T + r) * H) : nullptr;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int v = lt + k * kGroupThreads;
        if (v >= nv) continue;
        dy[v] = y[k];
        if (dr) dr[v] = res[k];
      }
    }
  }
  if (stamp) stamp[2] = now_ns();
  if (!barrier_flags(p.peer_flags, W, p.rank, p.err, 2, epoch, &bail, p.wait_ns)) return;  // every owner's rows landed
  for (int o = 0; o < W; ++o) {
    const int64_t e1 = min(static_cast<int64_t>(p.T), static_cast<int64_t>(o + 1) * p.Tc);
    for (int64_t r = static_cast<int64_t>(o) * p.Tc + slot0; r < e1; r += slots) {
      const uint4* gy = reinterpret_cast<const uint4*>(p.peer_gather[p.rank] + (par * p.max_T + r) * H);
      const uint4* gr = reinterpret_cast<const uint4*>(p.peer_gather_res[p.rank] + (par * p.max_T + r) * H);
      uint4 a[VPT], b[VPT];
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int v = lt + k * kGroupThreads;
        if (v >= nv) continue;
        a[k] = gy[v];
        if (p.gather_res && o != p.rank) b[k] = gr[v];
      }
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int v = lt + k * kGroupThreads;
        if (v >= nv) continue;
        reinterpret_cast<uint4*>(p.out + r * H)[v] = a[k];
        if (p.gather_res && o != p.rank) reinterpret_cast<uint4*>(p.residual + r * H)[v] = b[k];
      }
    }
  }
  if (stamp) stamp[3] = now_ns();
}

// Monotone 64-bit key of (value, global id): larger value first, then the
// lower id (first-occurrence argmax).  Float bits are mapped to an unsigned
// order (negative values bit-flipped, positive values with the sign bit set).
__device__ __forceinline__ unsigned long long argmax_key(float v, int64_t id) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) | (0xFFFFFFFFull - static_cast<unsigned long long>(id));
}

__global__ void __launch_bounds__(512) argmax_tp_kernel(ArgmaxParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  __shared__ float sb[16];
  __shared__ int si[16];
  __shared__ uint32_t s_epoch;
  __shared__ volatile int bail;
  if (threadIdx.x == 0) {
    s_epoch = ++p.counters[blockIdx.x];
    bail = 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const size_t par = epoch & 1u;
  const int W = p.world;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // 1. local argmax of each of this block's rows, key pushed to every rank
  for (int r = blockIdx.x; r < p.T; r += gridDim.x) {
    const __nv_bfloat16* row = p.logits + static_cast<int64_t>(r) * p.ld;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    const int nvec = p.V_local / 8;
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
      const uint4 u = reinterpret_cast<const uint4*>(row)[v];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        if (f.x > best) {
          best = f.x;
          idx = v * 8 + 2 * j;
        }
        if (f.y > best) {
          best = f.y;
          idx = v * 8 + 2 * j + 1;
        }
      }
    }
    for (int v = nvec * 8 + threadIdx.x; v < p.V_local; v += blockDim.x) {
      const float f = __bfloat162float(row[v]);
      if (f > best) {
        best = f;
        idx = v;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ob > best || (ob == best && oi < idx)) {
        best = ob;
        idx = oi;
      }
    }
    if (lane == 0) {
      sb[warp] = best;
      si[warp] = idx;
    }
    __syncthreads();
    if (warp == 0) {
      const int nw = blockDim.x >> 5;
      best = lane < nw ? sb[lane] : -INFINITY;
      idx = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ob > best || (ob == best && oi < idx)) {
          best = ob;
          idx = oi;
        }
      }
      // A row without a finite maximum keeps id 0 of this slice, as argmax_rows does.
      const unsigned long long key = argmax_key(best, p.vocab_offset + (idx == 0x7fffffff ? 0 : idx));
      if (lane < W) p.peer_keys[lane][(par * W + p.rank) * p.max_T + r] = key;
    }
    __syncthreads();
  }
  // 2. every rank's keys for this block's rows have landed here
  if (!barrier_flags(p.peer_flags, W, p.rank, p.err, 0, epoch, &bail, p.wait_ns)) return;
  // 3. best key over the ranks
  const unsigned long long* keys = p.peer_keys[p.rank] + par * W * static_cast<size_t>(p.max_T);
  for (int r = blockIdx.x; r < p.T; r += gridDim.x) {
    if (threadIdx.x == 0) {
      unsigned long long k = 0;
      for (int s = 0; s < W; ++s) {
        const unsigned long long ks = keys[static_cast<size_t>(s) * p.max_T + r];
        k = ks > k ? ks : k;
      }
      p.out[r] = static_cast<int64_t>(0xFFFFFFFFull - (k & 0xFFFFFFFFull));
    }
  }
}

}  // namespace comm
}  // namespace shk

using namespace shk::comm;

extern "C" int sh_argmax_tp(const ArgmaxParams* params, int num_blocks, cudaStream_t stream) {
  const ArgmaxParams& p = *params;
  if (p.world < 1 || p.world > SH_COMM_MAX_WORLD || p.T < 0 || p.T > p.max_T || p.V_local < 1) return -1;
  if ((reinterpret_cast<uintptr_t>(p.logits) & 15) || (p.ld * 2) % 16) return -2;
  if (p.vocab_offset < 0 || p.vocab_offset + p.V_local > 0xFFFFFFFFll) return -3;
  if (num_blocks < 1) num_blocks = 1;
  if (num_blocks > SH_COMM_MAX_BLOCKS) num_blocks = SH_COMM_MAX_BLOCKS;
  shk::launch(argmax_tp_kernel, dim3(num_blocks), dim3(512), 0, stream, p);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_allreduce(const ArParams* params, int num_blocks, cudaStream_t stream) {
  const ArParams& p = *params;
  if (p.world < 1 || p.world > SH_COMM_MAX_WORLD || p.H % 8 != 0 || p.T < 0 || p.T > p.max_T) return -1;
  if (p.fuse_norm && (p.residual == nullptr || p.weight == nullptr)) return -2;
  if (p.quant < 0 || p.quant > 2 || (p.quant && p.H % kQBlock != 0)) return -4;
  if (p.T == 0) return 0;
  if (num_blocks < 1) num_blocks = 1;
  if (num_blocks > SH_COMM_MAX_BLOCKS) num_blocks = SH_COMM_MAX_BLOCKS;
  const int nv = p.H / 8;
  const int vpt = (nv + kGroupThreads - 1) / kGroupThreads;
  const int threads = 4 * kGroupThreads;  // four rows per block
  auto run = [&](auto vpt_c) {
    constexpr int V = decltype(vpt_c)::value;
    if (p.quant)
      shk::launch(allreduce_kernel<V, true>, dim3(num_blocks), dim3(threads), 0, stream, p);
    else
      shk::launch(allreduce_kernel<V, false>, dim3(num_blocks), dim3(threads), 0, stream, p);
  };
  if (vpt == 1)
    run(std::integral_constant<int, 1>{});
  else if (vpt == 2)
    run(std::integral_constant<int, 2>{});
  else if (vpt <= 4)
    run(std::integral_constant<int, 4>{});
  else if (vpt <= 8)
    run(std::integral_constant<int, 8>{});
  else
    return -3;  // H > 8192
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_rs_norm_ag(const RsParams* params, int num_blocks, cudaStream_t stream) {
  const RsParams& p = *params;
  if (p.world < 1 || p.world > SH_COMM_MAX_WORLD || p.H % 8 != 0 || p.T < 0 || p.T > p.max_T || p.Tc < 1) return -1;
  if (!p.residual || !p.weight || !p.out || !p.rs_cnt || !p.targets || !p.counters) return -2;
  if (p.gather_res && !p.peer_gather_res[p.rank]) return -4;
  if (p.T == 0) return 0;
  if (num_blocks < 1) num_blocks = 1;
  if (num_blocks > SH_COMM_MAX_BLOCKS) num_blocks = SH_COMM_MAX_BLOCKS;
  const int nv = p.H / 8;
  const int vpt = (nv + kGroupThreads - 1) / kGroupThreads;
  const int threads = 4 * kGroupThreads;
  if (vpt == 1)
    shk::launch(rs_norm_ag_kernel<1>, dim3(num_blocks), dim3(threads), 0, stream, p);
  else if (vpt == 2)
    shk::launch(rs_norm_ag_kernel<2>, dim3(num_blocks), dim3(threads), 0, stream, p);
  else if (vpt <= 4)
    shk::launch(rs_norm_ag_kernel<4>, dim3(num_blocks), dim3(threads), 0, stream, p);
  else if (vpt <= 8)
    shk::launch(rs_norm_ag_kernel<8>, dim3(num_blocks), dim3(threads), 0, stream, p);
  else
    return -3;
  return static_cast<int>(cudaGetLastError());
}
