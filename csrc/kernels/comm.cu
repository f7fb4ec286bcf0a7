// Tensor-parallel all-reduce over NVLink peer memory, fused with the next
// layer's residual add + RMSNorm.
//
// Every rank's row-parallel GEMM writes its [T, H] partial straight into its
// symmetric buffer; this kernel then
//   one-shot (small T*H): every rank reads all peers' partials for its rows
//     (P2P loads over NVLink), sums them in rank order in fp32;
//   two-shot (large T*H): rank q reduces the rows it owns and stores the
//     bf16 sum into every rank's gather buffer (P2P stores), then each rank
//     reads the gathered sums from its own memory;
// and finishes with residual += sum, out = rms_norm(residual) * weight (or
// writes the plain sum).  Summation order is the same on every rank, so all
// ranks hold bit-identical results.
//
// Synchronisation: block b of every rank handles the same rows, so ranks only
// synchronise block-to-block.  A barrier is: __syncthreads, system-scope
// release store of the block's epoch into each peer's signal pad, then
// acquire loads of the peers' flags.  Epochs live in per-block device
// counters, so CUDA-graph replays stay aligned across ranks.  Each wait gives
// up after a time limit, records an error code in *err and skips the data
// phase (the step is then failed by the host; no trap, no hang).  The grid is
// at most one block per SM so every block is resident while it waits.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm.h"

namespace shk {
namespace comm {

constexpr uint64_t kTimeoutNs = 5000000000ull;  // 5 s
constexpr int kPhases = 3;

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
}

// Cross-rank barrier between same-index blocks. Returns false on timeout.
__device__ bool barrier(const ArParams& p, int phase, uint32_t epoch, volatile int* bail) {
  __syncthreads();
  if (threadIdx.x < p.world) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    st_release(flag_slot(p.peer_flags[threadIdx.x], phase, blockIdx.x, p.rank), epoch);
  }
  if (threadIdx.x < p.world) {
    const uint32_t* f = flag_slot(p.peer_flags[p.rank], phase, blockIdx.x, threadIdx.x);
    const uint64_t t0 = now_ns();
    while (static_cast<int32_t>(ld_acquire(f) - epoch) < 0) {
      if (*bail || now_ns() - t0 > kTimeoutNs) {
        *bail = 1;
        if (p.err) atomicCAS(p.err, 0, 100 + phase);
        break;
      }
    }
  }
  __syncthreads();
  return *bail == 0;
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

__device__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) t += red[i];
  __syncthreads();
  return t;
}

// residual += sum (bf16), out = rms_norm(residual) * w for one row; each
// thread owns the 8-element vectors v = threadIdx.x + k * blockDim.x.
template <int VPT>
__device__ void finish_row(const ArParams& p, int64_t r, float (*acc)[8], float* red) {
  const int nv = p.H / 8;
  float ss = 0.f;
  uint4 res[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = threadIdx.x + k * blockDim.x;
    if (v >= nv) continue;
    if (p.fuse_norm) {
      uint4 rv = reinterpret_cast<const uint4*>(p.residual + r * p.H)[v];
      float s[8];
      const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(rh[i]);
        s[2 * i] = f.x + acc[k][2 * i];
        s[2 * i + 1] = f.y + acc[k][2 * i + 1];
      }
      res[k] = pack8(s);  // the residual stream is stored in bf16
      const __nv_bfloat162* q = reinterpret_cast<const __nv_bfloat162*>(&res[k]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(q[i]);
        ss += f.x * f.x + f.y * f.y;
      }
      reinterpret_cast<uint4*>(p.residual + r * p.H)[v] = res[k];
    } else {
      reinterpret_cast<uint4*>(p.out + r * p.H)[v] = pack8(acc[k]);
    }
  }
  if (!p.fuse_norm) return;
  const float inv = rsqrtf(block_sum(ss, red) / p.H + p.eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = threadIdx.x + k * blockDim.x;
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
__global__ void __launch_bounds__(1024) allreduce_kernel(ArParams p) {
  __shared__ float red[32];
  __shared__ uint32_t s_epoch;
  __shared__ volatile int bail;
  if (threadIdx.x == 0) {
    s_epoch = ++p.counters[blockIdx.x];
    bail = 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int nv = p.H / 8;
  const int nb = gridDim.x;
  if (!barrier(p, 0, epoch, &bail)) return;  // every partial is written
  if (!p.two_shot) {
    for (int64_t r = blockIdx.x; r < p.T; r += nb) {
      float acc[VPT][8];
#pragma unroll
      for (int k = 0; k < VPT; ++k)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[k][i] = 0.f;
      for (int src = 0; src < p.world; ++src) {
        const uint4* in = reinterpret_cast<const uint4*>(p.peer_in[src] + r * p.H);
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
          const int v = threadIdx.x + k * blockDim.x;
          if (v < nv) add8(acc[k], in[v]);
        }
      }
      finish_row<VPT>(p, r, acc, red);
    }
    barrier(p, 2, epoch, &bail);  // peers are done reading this rank's partial
    return;
  }
  // Two-shot: rows r with r % nb == block; owner rank = (r / nb) % world.
  for (int64_t r = blockIdx.x; r < p.T; r += nb) {
    if ((r / nb) % p.world != p.rank) continue;
    float acc[VPT][8];
#pragma unroll
    for (int k = 0; k < VPT; ++k)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[k][i] = 0.f;
    for (int src = 0; src < p.world; ++src) {
      const uint4* in = reinterpret_cast<const uint4*>(p.peer_in[src] + r * p.H);
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int v = threadIdx.x + k * blockDim.x;
        if (v < nv) add8(acc[k], in[v]);
      }
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = threadIdx.x + k * blockDim.x;
      if (v >= nv) continue;
      const uint4 packed = pack8(acc[k]);
      for (int dst = 0; dst < p.world; ++dst) reinterpret_cast<uint4*>(p.peer_gather[dst] + r * p.H)[v] = packed;
    }
  }
  if (!barrier(p, 1, epoch, &bail)) return;  // every gathered sum has landed
  for (int64_t r = blockIdx.x; r < p.T; r += nb) {
    float acc[VPT][8];
    const uint4* g = reinterpret_cast<const uint4*>(p.peer_gather[p.rank] + r * p.H);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[k][i] = 0.f;
      const int v = threadIdx.x + k * blockDim.x;
      if (v < nv) add8(acc[k], g[v]);
    }
    finish_row<VPT>(p, r, acc, red);
  }
}

}  // namespace comm
}  // namespace shk

using namespace shk::comm;

extern "C" int sh_allreduce(const ArParams* params, int num_blocks, cudaStream_t stream) {
  const ArParams& p = *params;
  if (p.world < 1 || p.world > SH_COMM_MAX_WORLD || p.H % 8 != 0 || p.T < 0) return -1;
  if (p.fuse_norm && (p.residual == nullptr || p.weight == nullptr)) return -2;
  if (p.T == 0) return 0;
  if (num_blocks < 1) num_blocks = 1;
  if (num_blocks > SH_COMM_MAX_BLOCKS) num_blocks = SH_COMM_MAX_BLOCKS;
  const int nv = p.H / 8;
  int threads = 32;
  while (threads < nv && threads < 1024) threads <<= 1;
  const int vpt = (nv + threads - 1) / threads;
  if (vpt == 1)
    allreduce_kernel<1><<<num_blocks, threads, 0, stream>>>(p);
  else if (vpt == 2)
    allreduce_kernel<2><<<num_blocks, threads, 0, stream>>>(p);
  else if (vpt <= 4)
    allreduce_kernel<4><<<num_blocks, threads, 0, stream>>>(p);
  else
    return -3;  // H > 32768
  return static_cast<int>(cudaGetLastError());
}
