// Expert-parallel all-to-all over NVLink peer memory: dispatch of token rows
// to the ranks that hold their experts and combine of the expert outputs back
// to the token owners, with P2P stores issued from the kernels (replaces an
// all-gather of every token to every rank + reduce-scatter of the partials:
// a token row crosses NVLink only to ranks that host one of its top-k experts).
//
// dispatch (rank r, block b, tokens i = b, b + nblocks, ...): optionally
//   routes the token first from its router logits (the standalone router's
//   selection, moe_route.cuh; ids / weights also written for the combine);
//   for every rank d: route row (local expert id or -1, weight or 0) ->
//   d.ids / d.w [r*T + i]; for the ranks d hosting one of the token's experts:
//   x[i] -> d.x[r*T + i] (bf16), or with quant the row quantised once to
//   NVFP4 -> d.q / d.s / d.a [r*T + i] (3.55x fewer bytes; the receiving W4A4
//   expert GEMMs gather these codes directly); then a cross-rank barrier
//   between same-index blocks.
//   When the kernel finishes on d, every rank's rows have landed in d's buffers.
// experts: the grouped expert GEMMs of this rank over the [world*T, H] rows
//   (rows routed elsewhere have only -1 ids and are skipped).
// combine (rank d, block b, tokens i = b, b + nblocks, ...): for every source
//   rank r whose row r*T + i reached a local expert: y[r*T + i] ->
//   r.y_ret[d*T + i]; barrier; then out[i] = sum over the token's expert ranks
//   in rank order of y_ret[d*T + i] (fp32 accumulation, identical order on
//   every call).  Same-index blocks push and sum the same tokens, so the
//   block-to-block barrier covers exactly the rows each block reads.
//
// Buffers are single: a rank writes a peer's receive rows of call e+1 only
// after passing a barrier of call e+1 or e that the peer signals after it has
// finished reading call e's rows (dispatch writes follow the previous call's
// combine barrier, which each rank signals after its expert GEMMs; combine
// writes follow this call's dispatch barrier, signalled after the previous
// combine's sums).  Flags carry the per-block epoch, so no flag reset is
// needed, and the data pointers are the same every call (CUDA-graph safe).
// Every wait gives up after a time limit, records an error code and skips the
// remaining phases (no trap, no hang).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ep_a2a.h"
#include "moe_route.cuh"
#include "nvfp4_act.cuh"
#include "pdl.cuh"

namespace shk {
namespace ep {

using namespace shk::nvq;

constexpr uint64_t kTimeoutNs = 5000000000ull;  // 5 s
constexpr int kThreads = 512;

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
__device__ __forceinline__ uint32_t* flag_slot(uint32_t* base, int phase, int block, int src) {
  return base + (static_cast<size_t>(phase) * SH_EP_MAX_BLOCKS + block) * SH_EP_MAX_WORLD + src;
}

// Same-index blocks of all ranks meet; false on timeout (error recorded).
__device__ bool barrier(const EpParams& p, int phase, uint32_t epoch, volatile int* bail) {
  __syncthreads();  // every store of this block precedes the release below (cumulativity)
  if (threadIdx.x < p.world) st_release(flag_slot(p.peer_flags[threadIdx.x], phase, blockIdx.x, p.rank), epoch);
  if (threadIdx.x < p.world) {
    const uint32_t* f = flag_slot(p.peer_flags[p.rank], phase, blockIdx.x, threadIdx.x);
    const uint64_t t0 = now_ns();
    while (static_cast<int32_t>(ld_acquire(f) - epoch) < 0) {
      if (*bail || now_ns() - t0 > (p.wait_ns ? p.wait_ns : kTimeoutNs)) {
        *bail = 1;
        if (p.err) atomicCAS(p.err, 0, 200 + phase);
        break;
      }
    }
  }
  __syncthreads();
  return *bail == 0;
}

// Bit d set when one of the token's experts lives on rank d.
__device__ __forceinline__ uint32_t dest_mask(const EpParams& p, int64_t i) {
  uint32_t m = 0;
  for (int j = 0; j < p.k; ++j) {
    const int id = p.ids[i * p.k + j];
    if (id >= 0) m |= 1u << (id / p.e_local);
  }
  return m;
}

// Quantises token row i to NVFP4 in shared memory (codes then scales) and
// stores it into every destination rank's receive rows with 16-byte stores.
// qsm: H/2 + H/16 bytes of 16-byte aligned shared memory ([codes][scales]).
__device__ void quant_send(const EpParams& p, int64_t i, int64_t row, uint32_t m, uint8_t* qsm) {
  __shared__ float red[kThreads / 32];
  const int nblk = p.H / 16;
  const __nv_bfloat16* xr = p.x + i * p.H;
  float amax = 0.f;
  for (int b = threadIdx.x; b < nblk; b += kThreads) {
    float v[16];
    load16(xr + b * 16, v);
#pragma unroll
    for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  __syncthreads();  // the previous row's stores read qsm
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = 0.f;
  for (int w = 0; w < kThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  const float g = row_g(amax), g6 = __fdiv_rn(g, 6.f);
  for (int b = threadIdx.x; b < nblk; b += kThreads) {
    float v[16];
    load16(xr + b * 16, v);
    qsm[p.H / 2 + b] = quant16(v, g, g6, qsm + b * 8);
  }
  __syncthreads();
  const int nq = p.H / 32, ns = p.H / 256;  // 16-byte chunks of codes and of scales
  for (int d = 0; d < p.world; ++d) {
    if (!((m >> d) & 1u)) continue;
    uint4* dq = reinterpret_cast<uint4*>(p.peer_q[d] + row * (p.H / 2));
    uint4* ds = reinterpret_cast<uint4*>(p.peer_s[d] + row * (p.H / 16));
    for (int v = threadIdx.x; v < nq; v += kThreads) dq[v] = reinterpret_cast<const uint4*>(qsm)[v];
    for (int v = threadIdx.x; v < ns; v += kThreads) ds[v] = reinterpret_cast<const uint4*>(qsm + p.H / 2)[v];
    if (threadIdx.x == 0) p.peer_a[d][row] = __fdiv_rn(1.f, g);
  }
}

__global__ void __launch_bounds__(kThreads) ep_dispatch_kernel(EpParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  extern __shared__ __align__(16) uint8_t dsm[];  // [router scores 2E floats][NVFP4 row staging]
  __shared__ uint32_t s_epoch;
  __shared__ volatile int bail;
  __shared__ shk::route::Scratch rsc;
  __shared__ int tok_ids[SH_EP_MAX_K];
  __shared__ float tok_w[SH_EP_MAX_K];
  if (threadIdx.x == 0) {
    s_epoch = ++p.counters[blockIdx.x];
    bail = 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int nv = p.H / 8;
  const int64_t T = p.T;
  const int route_bytes = p.fused_route ? ((2 * p.route.E * 4 + 15) & ~15) : 0;
  for (int64_t i = blockIdx.x; i < T; i += gridDim.x) {
    const int64_t row = static_cast<int64_t>(p.rank) * T + i;  // this token's row on every rank
    __syncthreads();  // the previous token is done with tok_ids / tok_w and the staging
    if (p.fused_route) {  // route the token here: the same selection as the standalone router
      shk::route::route_token(p.route, i, shk::route::threads_for(p.route.E), reinterpret_cast<float*>(dsm), rsc);
      if (threadIdx.x < p.k) {
        tok_ids[threadIdx.x] = rsc.chosen_i[threadIdx.x];
        tok_w[threadIdx.x] = rsc.chosen_w[threadIdx.x];
        p.route.ids[i * p.k + threadIdx.x] = rsc.chosen_i[threadIdx.x];
        p.route.weights[i * p.k + threadIdx.x] = rsc.chosen_w[threadIdx.x];
      }
    } else if (threadIdx.x < p.k) {
      tok_ids[threadIdx.x] = p.ids[i * p.k + threadIdx.x];
      tok_w[threadIdx.x] = p.w[i * p.k + threadIdx.x];
    }
    __syncthreads();
    if (threadIdx.x < p.world * p.k) {
      const int d = threadIdx.x / p.k, j = threadIdx.x % p.k;
      const int id = tok_ids[j];
      const bool mine = id >= 0 && id / p.e_local == d;
      p.peer_ids[d][row * p.k + j] = mine ? id - d * p.e_local : -1;
      p.peer_w[d][row * p.k + j] = mine ? tok_w[j] : 0.f;
    }
    uint32_t m = 0;
    for (int j = 0; j < p.k; ++j)
      if (tok_ids[j] >= 0) m |= 1u << (tok_ids[j] / p.e_local);
    if (p.quant) {
      quant_send(p, i, row, m, dsm + route_bytes);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(p.x + i * p.H);
    for (int d = 0; d < p.world; ++d) {
      if (!((m >> d) & 1u)) continue;
      uint4* dst = reinterpret_cast<uint4*>(p.peer_x[d] + row * p.H);
      for (int v = threadIdx.x; v < nv; v += kThreads) dst[v] = src[v];
    }
  }
  barrier(p, 0, epoch, &bail);
}

__global__ void __launch_bounds__(kThreads) ep_combine_kernel(EpParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  __shared__ uint32_t s_epoch;
  __shared__ volatile int bail;
  if (threadIdx.x == 0) {
    s_epoch = p.counters[blockIdx.x];  // the epoch of this call's dispatch
    bail = 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int nv = p.H / 8;
  const int64_t T = p.T;
  const int32_t* my_ids = p.peer_ids[p.rank];
  // Push: row r*T + i of y goes back to its owner r when a local expert served it (unless the experts'
  // weighted sum already stored it there: ep_combine_push_kernel).
  for (int64_t i = blockIdx.x; i < T && !p.pushed; i += gridDim.x) {
    for (int r = 0; r < p.world; ++r) {
      const int64_t row = static_cast<int64_t>(r) * T + i;
      bool served = false;
      for (int j = 0; j < p.k; ++j) served |= my_ids[row * p.k + j] >= 0;
      if (!served) continue;
      const uint4* src = reinterpret_cast<const uint4*>(p.y + row * p.H);
      uint4* dst = reinterpret_cast<uint4*>(p.peer_y[r] + (static_cast<int64_t>(p.rank) * T + i) * p.H);
      for (int v = threadIdx.x; v < nv; v += kThreads) dst[v] = src[v];
    }
  }
  if (!barrier(p, 1, epoch, &bail)) return;
  // Sum the returned rows of each own token in rank order.
  const __nv_bfloat16* ret = p.peer_y[p.rank];
  for (int64_t i = blockIdx.x; i < T; i += gridDim.x) {
    const uint32_t m = dest_mask(p, i);
    for (int v = threadIdx.x; v < nv; v += kThreads) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int d = 0; d < p.world; ++d) {
        if (!((m >> d) & 1u)) continue;
        const uint4 u = reinterpret_cast<const uint4*>(ret + (static_cast<int64_t>(d) * T + i) * p.H)[v];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          acc[2 * e] += f.x;
          acc[2 * e + 1] += f.y;
        }
      }
      uint4 o;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) oh[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
      reinterpret_cast<uint4*>(p.out + i * p.H)[v] = o;
    }
  }
}

// The experts' weighted per-token sum of the received rows, stored straight into
// the owners' return rows: the same arithmetic as moe.cu combine_kernel (fp32
// accumulation in slot order, one bf16 rounding), so the owner's sum is
// bit-identical to combine_kernel followed by ep_combine_kernel's push.  Rows
// no local expert served are not stored.  Every thread fences at system
// scope after its stores, and the following ep_combine_kernel (pushed = 1)
// starts after this grid has completed, so its barrier orders these stores
// before the owners read them.
__global__ void __launch_bounds__(kThreads) ep_combine_push_kernel(EpParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  // A dispatch barrier of this call that timed out leaves the peers' state
  // unknown (one may still be reading the previous call's return rows):
  // store nothing into peer memory then.  The error is already recorded.
  if (p.err && *reinterpret_cast<volatile const int*>(p.err) != 0) return;
  const int64_t T = p.T;
  const int32_t* my_ids = p.peer_ids[p.rank];
  for (int64_t row = blockIdx.x; row < static_cast<int64_t>(p.world) * T; row += gridDim.x) {
    bool served = false;
    for (int j = 0; j < p.k; ++j) served |= my_ids[row * p.k + j] >= 0;
    if (!served) continue;
    const int r = static_cast<int>(row / T);
    const int64_t i = row % T;
    __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(p.peer_y[r] + (static_cast<int64_t>(p.rank) * T + i) * p.H);
    for (int e = threadIdx.x; e < p.H / 2; e += kThreads) {
      float2 acc = make_float2(0.f, 0.f);
      for (int j = 0; j < p.k; ++j) {
        const int pos = p.sorted_pos[row * p.k + j];
        if (pos < 0) continue;
        const float wj = p.w_local[row * p.k + j];
        const float2 v = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(p.ys + static_cast<int64_t>(pos) * p.H)[e]);
        acc.x += wj * v.x;
        acc.y += wj * v.y;
      }
      dst[e] = __floats2bfloat162_rn(acc.x, acc.y);
    }
  }
  __threadfence_system();  // this thread's peer stores are visible system-wide before the grid completes
}

}  // namespace ep
}  // namespace shk

using namespace shk::ep;

static int ep_check(const EpParams& p) {
  if (p.world < 1 || p.world > SH_EP_MAX_WORLD || p.H % 8 != 0 || p.T < 0 || p.T > p.max_T) return -1;
  if (p.k < 1 || p.k > SH_EP_MAX_K || p.world * p.k > kThreads || p.e_local < 1) return -2;
  if (p.quant && (p.H % 256 != 0 || p.H / 2 + p.H / 16 > 24 * 1024)) return -3;  // 16-byte scale rows
  if (p.fused_route) {
    const RouteParams& r = p.route;
    if (r.k != p.k || r.E < r.k || r.E > 2048 || !r.logits || !r.ids || !r.weights || r.ids != p.ids) return -4;
    if (r.sigmoid_grouped && (r.n_groups < 1 || r.E % r.n_groups || r.n_groups > 64)) return -4;
  }
  return 0;
}

extern "C" int sh_ep_dispatch(const EpParams* params, int num_blocks, cudaStream_t stream) {
  const int rc = ep_check(*params);
  if (rc) return rc;
  if (params->T == 0) return 0;
  num_blocks = num_blocks < 1 ? 1 : (num_blocks > SH_EP_MAX_BLOCKS ? SH_EP_MAX_BLOCKS : num_blocks);
  const size_t smem = (params->fused_route ? ((2 * params->route.E * 4 + 15) & ~15) : 0) +
                      (params->quant ? static_cast<size_t>(params->H / 2 + params->H / 16) : 0);
  shk::launch(ep_dispatch_kernel, dim3(num_blocks), dim3(kThreads), smem, stream, *params);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_ep_combine(const EpParams* params, int num_blocks, cudaStream_t stream) {
  const int rc = ep_check(*params);
  if (rc) return rc;
  if (params->T == 0) return 0;
  num_blocks = num_blocks < 1 ? 1 : (num_blocks > SH_EP_MAX_BLOCKS ? SH_EP_MAX_BLOCKS : num_blocks);
  shk::launch(ep_combine_kernel, dim3(num_blocks), dim3(kThreads), 0, stream, *params);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_ep_combine_push(const EpParams* params, int num_blocks, cudaStream_t stream) {
  const int rc = ep_check(*params);
  if (rc) return rc;
  if (!params->ys || !params->sorted_pos || !params->w_local) return -5;
  if (params->T == 0) return 0;
  num_blocks = num_blocks < 1 ? 1 : (num_blocks > SH_EP_MAX_BLOCKS ? SH_EP_MAX_BLOCKS : num_blocks);
  shk::launch(ep_combine_push_kernel, dim3(num_blocks), dim3(kThreads), 0, stream, *params);
  return static_cast<int>(cudaGetLastError());
}
