// Host KV tier (HiSparse) for sparse-attention decode: the full MLA latent cache of a layer stays in host
// memory that the GPU maps, and each request slot owns H device ("hot") rows of that layer.  Before the
// MLA kernel of a decode step, one CTA per request resolves the request's top-k key positions:
//
//   0. positions the step writes lose their hot copy (a rejected draft's position is rewritten next step,
//      so a resident row would be stale);
//   1. a key whose position is resident stamps its row with this step's tick (a hit); a key that is not
//      claims its position (pos2slot -1 -> -2), so keys shared by the request's query tokens fetch once;
//   2. victims are chosen least recently used first among rows no key of this step uses (free rows
//      first), through a 256-bin histogram of row ages;
//   3. each claimed position takes a victim row, whose old position loses residency;
//   4. the fetched rows are copied from host memory with 16-byte loads, four rows per warp in flight;
//   5. the request's top-k list is rewritten as hot-row indices, in the same order, and its hot
//      block-table row and a causal-safe length are written, so the MLA kernel reads the hot rows as an
//      ordinary paged cache.
//
// The keys, their order and the rows' bytes are those of the host cache, so attention over the hot rows
// is bit-identical to attention over the host cache.  More distinct keys in one step than H hot rows is an
// error (601 in *err; the excess keys are dropped): H is sized as (verify width) x top-k or more.
//
// Reference parity: suffix_hisparse_resolve / suffix_hisparse_invalidate, the hot-buffer residency
// resolver over a host-pinned KV pool (reference: sm120/hisparse_mtp_patch/own_resolver.py:200-690).
#include <cuda_runtime.h>
#include <stdint.h>

#include "hisparse.h"
#include "pdl.cuh"

namespace shk {
namespace hs {

constexpr int THREADS = 1024;
constexpr int BINS = 256;
constexpr int UNROLL = 4;  // independent entries (or rows) per thread (or warp) and pass

__device__ __forceinline__ int row_age(int32_t owner, int32_t stamp, int tick) {
  return owner < 0 ? BINS - 1 : min(BINS - 1, max(1, tick - stamp));
}

__global__ void __launch_bounds__(THREADS) resolve_kernel(HsParams p) {
  shk::pdl_trigger();
  shk::pdl_wait();
  extern __shared__ int32_t sm[];
  int32_t* miss = sm;           // [H] positions to fetch
  int32_t* vict = sm + p.H;     // [H] their rows
  int32_t* hist = sm + 2 * p.H; // [BINS] rows per age
  __shared__ int nmiss, nvict, tb, tb_need, tb_taken, overflow, hits;
  const int b = blockIdx.x, tid = threadIdx.x;
  const int64_t slot = p.state_slots[b];
  int32_t* p2s = p.pos2slot + slot * p.P;
  int32_t* s2p = p.slot2pos + slot * p.H;
  int32_t* stp = p.stamp + slot * p.H;
  const int64_t qs = p.q_start[b], qe = p.q_start[b + 1], ql = qe - qs, seq = p.seq_lens[b];
  const int tick = p.clock[slot] + 1;
  if (tid == 0) nmiss = nvict = tb_taken = overflow = hits = 0;
  for (int i = tid; i < BINS; i += THREADS) hist[i] = 0;
  // 0. written positions
  for (int64_t t = qs + tid; t < qe; t += THREADS) {
    const int64_t pos = p.positions[t];
    if (p.slot_mapping[t] < 0 || pos < 0 || pos >= p.P) continue;
    const int32_t h = p2s[pos];
    if (h >= 0) {
      p2s[pos] = -1;
      s2p[h] = -1;
    }
  }
  __syncthreads();
  // 1. hits and claimed misses
  const int64_t n = ql * p.K;
  const int32_t* tk = p.topk + qs * p.K;
  int my_hits = 0;
  // UNROLL entries per thread per pass: their positions, then their residency entries, load back to back
  for (int64_t e0 = tid; e0 < n; e0 += UNROLL * THREADS) {
    int32_t pos[UNROLL], h[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t e = e0 + u * THREADS;
      pos[u] = -1;
      if (e < n) {
        const int32_t q = tk[e];
        if (q >= 0 && q <= seq - ql + e / p.K && q < p.P) pos[u] = q;
      }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) h[u] = pos[u] >= 0 ? p2s[pos[u]] : -1;
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      if (pos[u] < 0) continue;
      if (h[u] >= 0) {
        stp[h[u]] = tick;
        ++my_hits;
        continue;
      }
      if (atomicCAS(&p2s[pos[u]], -1, -2) == -1) {
        const int j = atomicAdd(&nmiss, 1);
        if (j < p.H) {
          miss[j] = pos[u];
        } else {
          p2s[pos[u]] = -1;
          overflow = 1;
        }
      }
    }
  }
  if (my_hits) atomicAdd(&hits, my_hits);
  __syncthreads();
  const int need = min(nmiss, p.H);
  // 2. victims: all rows older than the threshold age, then enough rows of that age
  if (need > 0) {
    for (int h0 = tid; h0 < p.H; h0 += UNROLL * THREADS) {
      int32_t o[UNROLL], st[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int h = h0 + u * THREADS;
        o[u] = h < p.H ? s2p[h] : 0;
        st[u] = h < p.H ? stp[h] : tick;
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u)
        if (!(o[u] >= 0 && st[u] == tick)) atomicAdd(&hist[row_age(o[u], st[u], tick)], 1);
    }
    __syncthreads();
    if (tid == 0) {
      int acc = 0, bin = BINS - 1;
      for (; bin >= 1; --bin) {
        if (acc + hist[bin] >= need) break;
        acc += hist[bin];
      }
      tb = bin;
      tb_need = need - acc;
    }
    __syncthreads();
    for (int h0 = tid; h0 < p.H; h0 += UNROLL * THREADS) {
      int32_t o[UNROLL], st[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int h = h0 + u * THREADS;
        o[u] = h < p.H ? s2p[h] : 0;
        st[u] = h < p.H ? stp[h] : tick;
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        if (o[u] >= 0 && st[u] == tick) continue;  // in use this step, or past the rows (o 0, stamp tick)
        const int age = row_age(o[u], st[u], tick);
        if (age > tb || (age == tb && atomicAdd(&tb_taken, 1) < tb_need)) {
          const int j = atomicAdd(&nvict, 1);
          if (j < need) vict[j] = h0 + u * THREADS;
        }
      }
    }
    __syncthreads();
  }
  // 3. assignment
  const int nv = min(nvict, need);
  for (int j = tid; j < need; j += THREADS) {
    const int32_t pos = miss[j];
    if (j < nv) {
      const int32_t h = vict[j];
      const int32_t old = s2p[h];
      if (old >= 0) p2s[old] = -1;
      s2p[h] = pos;
      stp[h] = tick;
      p2s[pos] = h;
    } else {
      p2s[pos] = -1;
      overflow = 1;
    }
  }
  __syncthreads();
  // 4. fetch rows from host memory
  {
    const int warp = tid >> 5, lane = tid & 31, chunks = p.row_bytes >> 4;
    const int32_t* bt = p.block_tables + static_cast<int64_t>(b) * p.bt_stride;
    // a warp moves UNROLL rows per pass: their block-table entries, then all their 16-byte chunks, in flight
    // together (host-memory reads are the longest latency here)
    for (int j0 = warp; j0 < nv; j0 += UNROLL * (THREADS / 32)) {
      int64_t crow[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int j = j0 + u * (THREADS / 32);
        crow[u] = -1;
        if (j < nv) {
          const int32_t pos = miss[j];
          crow[u] = static_cast<int64_t>(bt[pos >> 6]) * 64 + (pos & 63);
        }
      }
      for (int c = lane; c < chunks; c += 32) {
        uint4 v[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u)
          if (crow[u] >= 0) v[u] = reinterpret_cast<const uint4*>(p.cold + crow[u] * p.row_bytes)[c];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u)
          if (crow[u] >= 0)
            reinterpret_cast<uint4*>(p.hot + (slot * p.H + vict[j0 + u * (THREADS / 32)]) * p.row_bytes)[c] = v[u];
      }
    }
  }
  // 5. rewritten top-k, hot block-table row, causal-safe length
  int32_t* out = p.topk_out + qs * p.K;
  for (int64_t e0 = tid; e0 < n; e0 += UNROLL * THREADS) {
    int32_t pos[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t e = e0 + u * THREADS;
      pos[u] = -1;
      if (e < n) {
        const int32_t q = tk[e];
        if (q >= 0 && q <= seq - ql + e / p.K && q < p.P) pos[u] = q;
      }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int64_t e = e0 + u * THREADS;
      if (e < n) out[e] = pos[u] >= 0 ? max(p2s[pos[u]], -1) : -1;
    }
  }
  const int hb = p.H / 64;
  for (int j = tid; j < hb; j += THREADS) p.hot_bt[static_cast<int64_t>(b) * hb + j] = static_cast<int32_t>(slot * hb + j);
  if (tid == 0) {
    p.hot_seq[b] = p.H + ql;
    p.clock[slot] = tick;
    if (overflow && p.err) atomicCAS(p.err, 0, 601);
    if (p.stats) {
      atomicAdd(reinterpret_cast<unsigned long long*>(p.stats), static_cast<unsigned long long>(hits));
      atomicAdd(reinterpret_cast<unsigned long long*>(p.stats + 1), static_cast<unsigned long long>(nv));
    }
  }
}

__global__ void reset_kernel(int32_t* pos2slot, int32_t* slot2pos, int32_t* stamp, int32_t* clock,
                             const int64_t* slots, int num_slots, int H, int P) {
  const int64_t slot = slots[blockIdx.x];
  const int64_t l = blockIdx.y;
  if (slot < 0 || slot >= num_slots) return;
  int32_t* p2s = pos2slot + (l * num_slots + slot) * P;
  for (int i = threadIdx.x; i < P; i += blockDim.x) p2s[i] = -1;
  int32_t* s2p = slot2pos + (l * num_slots + slot) * H;
  int32_t* stp = stamp + (l * num_slots + slot) * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    s2p[i] = -1;
    stp[i] = 0;
  }
  if (threadIdx.x == 0) clock[l * num_slots + slot] = 0;
}

}  // namespace hs
}  // namespace shk

extern "C" int sh_hisparse_resolve(const HsParams* p, cudaStream_t stream) {
  if (p->B <= 0) return 0;
  if (p->H <= 0 || p->H % 64 != 0 || p->H > 16384 || p->row_bytes % 16 != 0 || p->K <= 0) return -1;
  const int smem = (2 * p->H + shk::hs::BINS) * 4;
  static int ready = 0;
  if (ready < smem) {
    const cudaError_t e =
        cudaFuncSetAttribute(shk::hs::resolve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 16384 * 4 + 1024);
    if (e != cudaSuccess) return static_cast<int>(e);
    ready = 2 * 16384 * 4 + 1024;
  }
  shk::launch(shk::hs::resolve_kernel, dim3(p->B), dim3(shk::hs::THREADS), smem, stream, *p);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int sh_hisparse_reset(int32_t* pos2slot, int32_t* slot2pos, int32_t* stamp, int32_t* clock,
                                 const int64_t* slots, int n, int layers, int num_slots, int H, int P,
                                 cudaStream_t stream) {
  if (n <= 0 || layers <= 0) return 0;
  shk::hs::reset_kernel<<<dim3(n, layers), 256, 0, stream>>>(pos2slot, slot2pos, stamp, clock, slots, num_slots, H,
                                                               P);
  return static_cast<int>(cudaGetLastError());
}
