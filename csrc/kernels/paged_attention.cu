// Paged GQA attention for prefill, decode and speculative verify.
//
// One CTA owns one (request, kv head, 64-row query tile).  A query tile packs
// (token, q-head-of-this-group) rows: row r -> token r / G, head h*G + r % G,
// so the G query heads sharing a kv head (and the k+1 verify tokens of a
// request) read every K/V page exactly once.  K/V pages are 64 tokens of a
// [num_blocks, kv_heads, 64, D] cache, streamed through a two-stage cp.async
// ring into XOR-swizzled shared memory; QK^T and PV run on bf16 tensor-core
// tiles with fp32 accumulation and an exp2 online softmax.  Causality is by
// absolute position: the query token at position p sees keys [0, p].
// Query rows are read in place from the fused QKV projection output.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"

namespace shk {

constexpr int kAttnRows = 64;  // query rows per CTA (4 warps x 16)
constexpr int kAttnKeys = 64;  // keys per page / tile

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of 16-byte chunk `c` of row `r` in a swizzled [rows][D] bf16 tile.
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * D * 2 + ((c ^ (r & 7)) << 4));
}

template <int D>
__device__ __forceinline__ void load_page(uint8_t* dst, const __nv_bfloat16* src, int valid_keys) {
  constexpr int CH = D / 8;  // 16-byte chunks per row
  for (int c = threadIdx.x; c < kAttnKeys * CH; c += blockDim.x) {
    const int r = c / CH, ch = c % CH;
    cp_async16(dst + swz<D>(r, ch), src + r * D + ch * 8, r < valid_keys);
  }
}

template <int D>
__global__ void __launch_bounds__(128) paged_attention_kernel(
    __nv_bfloat16* __restrict__ out, int64_t out_stride_tok, const __nv_bfloat16* __restrict__ q,
    int64_t q_stride_tok, const __nv_bfloat16* __restrict__ k_cache, const __nv_bfloat16* __restrict__ v_cache,
    const int32_t* __restrict__ block_tables, int64_t bt_stride, const int64_t* __restrict__ seq_lens,
    const int64_t* __restrict__ q_start, const int32_t* __restrict__ tile_req, const int32_t* __restrict__ tile_row0,
    int hq, int hk, float scale_log2) {
  constexpr int CH = D / 8;
  constexpr int KSTEPS = D / 16;
  constexpr int DT = D / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK[2] = {smem + kAttnRows * D * 2, smem + kAttnRows * D * 2 + kAttnKeys * D * 2};
  uint8_t* sV[2] = {smem + kAttnRows * D * 2 + 2 * kAttnKeys * D * 2,
                    smem + kAttnRows * D * 2 + 3 * kAttnKeys * D * 2};

  const int b = tile_req[blockIdx.x];
  const int row0 = tile_row0[blockIdx.x];
  const int h = blockIdx.y;
  const int G = hq / hk;
  const int64_t qs = q_start[b];
  const int q_len = static_cast<int>(q_start[b + 1] - qs);
  const int64_t seq_len = seq_lens[b];
  const int64_t ctx0 = seq_len - q_len;  // absolute position of the first query token
  const int rows_valid = min(kAttnRows, q_len * G - row0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;

  // Query rows -> smem (zero-filled past the valid rows).
  for (int c = threadIdx.x; c < kAttnRows * CH; c += blockDim.x) {
    const int r = c / CH, ch = c % CH;
    const bool ok = r < rows_valid;
    const int rr = ok ? row0 + r : row0;
    const int tok = rr / G, head = h * G + rr % G;
    cp_async16(sQ + swz<D>(r, ch), q + (qs + tok) * q_stride_tok + (int64_t)head * D + ch * 8, ok);
  }
  const int last_row = row0 + rows_valid - 1;
  const int64_t kv_end = min(seq_len, ctx0 + last_row / G + 1);  // keys any row of this tile may see
  const int ntiles = static_cast<int>((kv_end + kAttnKeys - 1) / kAttnKeys);
  const int32_t* bt = block_tables + (int64_t)b * bt_stride;
  auto page_ptr = [&](const __nv_bfloat16* cache, int j) {
    return cache + ((int64_t)bt[j] * hk + h) * (int64_t)kAttnKeys * D;
  };
  if (ntiles > 0) {
    const int vk = static_cast<int>(kv_end < kAttnKeys ? kv_end : (int64_t)kAttnKeys);
    load_page<D>(sK[0], page_ptr(k_cache, 0), vk);
    load_page<D>(sV[0], page_ptr(v_cache, 0), vk);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  const bool warp_active = warp * 16 < rows_valid;
  uint32_t qf[KSTEPS][4];
  if (warp_active) {
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      const int r = warp * 16 + (lane & 15);
      const int ch = 2 * kk + (lane >> 4);
      ldsm_x4(smem_u32(sQ) + swz<D>(r, ch), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  }
  // Absolute positions of this thread's two rows (-1 = padding row).
  const int ra = warp * 16 + g, rb = ra + 8;
  const int64_t pa = ra < rows_valid ? ctx0 + (row0 + ra) / G : -1;
  const int64_t pb = rb < rows_valid ? ctx0 + (row0 + rb) / G : -1;

  float o[DT][4];
#pragma unroll
  for (int i = 0; i < DT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;

  for (int j = 0; j < ntiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < ntiles) {
      const int vk = static_cast<int>(min((int64_t)kAttnKeys, kv_end - (int64_t)(j + 1) * kAttnKeys));
      load_page<D>(sK[buf ^ 1], page_ptr(k_cache, j + 1), vk);
      load_page<D>(sV[buf ^ 1], page_ptr(v_cache, j + 1), vk);
    }
    cp_async_commit();
    if (warp_active) {
      float s[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
      const uint32_t kb = smem_u32(sK[buf]);
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int ch = 2 * kk + ((lane >> 3) & 1);
          ldsm_x4(kb + swz<D>(key, ch), b0, b1, b2, b3);
          mma_bf16(s[2 * np], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
          mma_bf16(s[2 * np + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
        }
      }
      // Scale, mask, online softmax.
      const int64_t kbase = (int64_t)j * kAttnKeys;
      const bool edge = kbase + kAttnKeys - 1 > min(pa, pb) || pa < 0 || pb < 0;
      float mx_a = m_a, mx_b = m_b;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int64_t kp = kbase + nt * 8 + 2 * t4 + e;
          float va = s[nt][e] * scale_log2, vb = s[nt][2 + e] * scale_log2;
          if (edge) {
            if (kp > pa) va = -INFINITY;
            if (kp > pb) vb = -INFINITY;
          }
          s[nt][e] = va;
          s[nt][2 + e] = vb;
          mx_a = fmaxf(mx_a, va);
          mx_b = fmaxf(mx_b, vb);
        }
      }
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
      const float base_a = mx_a == -INFINITY ? 0.f : mx_a;
      const float base_b = mx_b == -INFINITY ? 0.f : mx_b;
      const float alpha_a = exp2f(m_a - base_a), alpha_b = exp2f(m_b - base_b);
      m_a = mx_a;
      m_b = mx_b;
      float sum_a = 0.f, sum_b = 0.f;
      uint32_t pf[4][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float p0 = exp2f(s[nt][0] - base_a), p1 = exp2f(s[nt][1] - base_a);
        const float p2 = exp2f(s[nt][2] - base_b), p3 = exp2f(s[nt][3] - base_b);
        sum_a += p0 + p1;
        sum_b += p2 + p3;
        const int kc = nt >> 1, hi = nt & 1;
        pf[kc][hi * 2 + 0] = pack_bf16(p0, p1);
        pf[kc][hi * 2 + 1] = pack_bf16(p2, p3);
      }
      l_a = l_a * alpha_a + sum_a;
      l_b = l_b * alpha_b + sum_b;
#pragma unroll
      for (int dt = 0; dt < DT; ++dt) {
        o[dt][0] *= alpha_a;
        o[dt][1] *= alpha_a;
        o[dt][2] *= alpha_b;
        o[dt][3] *= alpha_b;
      }
      const uint32_t vb_ = smem_u32(sV[buf]);
#pragma unroll
      for (int kc = 0; kc < 4; ++kc) {
        // A fragment order: a0 (row g, keys lo), a1 (row g+8, keys lo), a2 (row g, keys hi), a3 (row g+8, hi).
        const uint32_t a0 = pf[kc][0], a1 = pf[kc][1], a2 = pf[kc][2], a3 = pf[kc][3];
#pragma unroll
        for (int dp = 0; dp < DT / 2; ++dp) {
          uint32_t b0, b1, b2, b3;
          const int key = kc * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int ch = 2 * dp + (lane >> 4);
          ldsm_x4_t(vb_ + swz<D>(key, ch), b0, b1, b2, b3);
          mma_bf16(o[2 * dp], a0, a1, a2, a3, b0, b1);
          mma_bf16(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    cp_async_wait<0>();
    __syncthreads();
  }
  if (!warp_active) return;
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f;
  const float inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
  if (ra < rows_valid) {
    const int rr = row0 + ra;
    __nv_bfloat16* dst = out + (qs + rr / G) * out_stride_tok + (int64_t)(h * G + rr % G) * D;
#pragma unroll
    for (int dt = 0; dt < DT; ++dt)
      *reinterpret_cast<__nv_bfloat162*>(dst + dt * 8 + 2 * t4) =
          __floats2bfloat162_rn(o[dt][0] * inv_a, o[dt][1] * inv_a);
  }
  if (rb < rows_valid) {
    const int rr = row0 + rb;
    __nv_bfloat16* dst = out + (qs + rr / G) * out_stride_tok + (int64_t)(h * G + rr % G) * D;
#pragma unroll
    for (int dt = 0; dt < DT; ++dt)
      *reinterpret_cast<__nv_bfloat162*>(dst + dt * 8 + 2 * t4) =
          __floats2bfloat162_rn(o[dt][2] * inv_b, o[dt][3] * inv_b);
  }
}

}  // namespace shk

using namespace shk;

// q: [T, >= hq*D] view (row stride q_stride), out: [T, hq*D] (row stride).
// tile_req / tile_row0: int32 [num_tiles] q-tile schedule (see plan_attention_tiles).
void paged_attention(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                     torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor q_start,
                     torch::Tensor tile_req, torch::Tensor tile_row0, int64_t hq, double scale) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k_cache.scalar_type() == at::kBFloat16, "bf16 attention");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == kAttnKeys, "cache must be [blocks, hk, 64, D]");
  TORCH_CHECK(q.stride(-1) == 1 && out.stride(-1) == 1, "q/out innermost stride 1");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kLong &&
                  q_start.scalar_type() == at::kLong && tile_req.scalar_type() == at::kInt,
              "attention index dtypes");
  const int hk = k_cache.size(1), d = k_cache.size(3);
  TORCH_CHECK(hq % hk == 0, "hq must be a multiple of hk");
  const int ntiles = tile_req.numel();
  if (ntiles == 0) return;
  const float scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  auto stream = at::cuda::getCurrentCUDAStream();
  dim3 grid(ntiles, hk);
  auto launch = [&](auto kernel, int D) {
    const int smem = (kAttnRows + 4 * kAttnKeys) * D * 2;
    SH_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kernel<<<grid, 128, smem, stream>>>((__nv_bfloat16*)out.data_ptr(), out.stride(0),
                                        (const __nv_bfloat16*)q.data_ptr(), q.stride(0),
                                        (const __nv_bfloat16*)k_cache.data_ptr(),
                                        (const __nv_bfloat16*)v_cache.data_ptr(), block_tables.data_ptr<int32_t>(),
                                        block_tables.stride(0), seq_lens.data_ptr<int64_t>(),
                                        q_start.data_ptr<int64_t>(), tile_req.data_ptr<int32_t>(),
                                        tile_row0.data_ptr<int32_t>(), (int)hq, hk, scale_log2);
  };
  if (d == 128)
    launch(paged_attention_kernel<128>, 128);
  else if (d == 64)
    launch(paged_attention_kernel<64>, 64);
  else if (d == 256)
    launch(paged_attention_kernel<256>, 256);
  else
    TORCH_CHECK(false, "paged_attention: head_dim must be 64, 128 or 256");
  SH_CUDA_CHECK(cudaGetLastError());
}
