// Greedy sampling and fused draft verification.
//
//  * argmax_rows: first-occurrence argmax per logits row (matches
//    torch.argmax), one CTA per row, 16-byte vector loads.
//  * spec_verify: the on-device greedy verify + commit step.  For request b
//    the verify window holds [x_L, d_1..d_k] at positions L..L+k and the
//    target's argmax t_0..t_k.  accept a = longest prefix with d_i == t_{i-1}
//    (a -1 pad never matches); emitted tokens are d_1..d_a followed by the
//    bonus t_a; the committed length becomes L + a + 1 and the next window
//    starts with t_a.  Stale cache entries past the committed length are
//    never read (attention is bounded by the sequence length) and are
//    overwritten by the next window, so no cache copy is needed.  Semantics
//    of the accept run match the reference's greedy verify oracle
//    (reference: src/verify_fusion.rs:48-113).
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "pdl.cuh"

namespace shk {

template <typename T, int VEC>
__global__ void argmax_rows_kernel(int64_t* __restrict__ out, const T* __restrict__ logits, int64_t vocab,
                                   int64_t stride) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const T* row = logits + (int64_t)blockIdx.x * stride;
  float best = -INFINITY;
  int64_t idx = 0x7fffffffffffffffll;
  const int64_t nvec = vocab / VEC;
  for (int64_t v = threadIdx.x; v < nvec; v += blockDim.x) {
    T buf[VEC];
    *reinterpret_cast<float4*>(buf) = reinterpret_cast<const float4*>(row)[v];
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float f = to_f(buf[j]);
      if (f > best) {  // strict: earliest index wins within a thread's ascending walk
        best = f;
        idx = v * VEC + j;
      }
    }
  }
  for (int64_t v = nvec * VEC + threadIdx.x; v < vocab; v += blockDim.x) {
    const float f = to_f(row[v]);
    if (f > best || (f == best && v < idx)) {
      best = f;
      idx = v;
    }
  }
  // Reduce (max value, then smallest index).
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) {
      best = ob;
      idx = oi;
    }
  }
  __shared__ float sb[32];
  __shared__ int64_t si[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sb[warp] = best;
    si[warp] = idx;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -INFINITY;
    idx = lane < nw ? si[lane] : 0x7fffffffffffffffll;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ob > best || (ob == best && oi < idx)) {
        best = ob;
        idx = oi;
      }
    }
    if (lane == 0) out[blockIdx.x] = idx == 0x7fffffffffffffffll ? 0 : idx;
  }
}

// One thread per request.  Row strides (elements) let the step verify the
// first W columns of wider static buffers.
__global__ void spec_verify_kernel(const int64_t* __restrict__ draft, const int64_t* __restrict__ target,
                                   int64_t* __restrict__ seq_lens, int64_t* __restrict__ out_tokens,
                                   int32_t* __restrict__ accept, int64_t* __restrict__ next_token, int batch, int k,
                                   int64_t ld_d, int64_t ld_t, int64_t ld_o) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const int64_t* d = draft + (int64_t)b * ld_d;
  const int64_t* t = target + (int64_t)b * ld_t;
  int a = 0;
  while (a < k && d[a] >= 0 && d[a] == t[a]) ++a;
  int64_t* o = out_tokens + (int64_t)b * ld_o;
  for (int i = 0; i < a; ++i) o[i] = d[i];
  o[a] = t[a];
  for (int i = a + 1; i <= k; ++i) o[i] = -1;
  accept[b] = a;
  next_token[b] = t[a];
  seq_lens[b] += a + 1;
}

// Async-scheduling advance (one thread per request): builds the next verify
// window on the device from this step's results and a host candidate computed
// one step earlier.  cand [B, L] (row b: C_b[0:clen_b]) was anchored at the
// history length before this step; the step accepted a_b drafts and appended
// o = a_b + 1 tokens out[b, 0:o].  If C_b[0:o] == out[b, 0:o] the next drafts
// are C_b[o : o+k] (positions < clen_b; -1 = no draft), else none.  With
// native != nullptr (hybrid) the native drafts native[b, 0:k] are used unless
// at least hyb_min candidate drafts are real.  win[b] = [next_token[b],
// drafts]; seq[b] = seq_new[b]; real[b] = number of candidate drafts used.
// Rows b >= real_batch (bucket padding) are reset to the scratch window
// (zeros, length 0).
__global__ void spec_advance_kernel(const int64_t* __restrict__ out_tokens, const int32_t* __restrict__ accept,
                                    const int64_t* __restrict__ next_token, const int64_t* __restrict__ seq_new,
                                    const int64_t* __restrict__ cand, const int32_t* __restrict__ clen,
                                    const int64_t* __restrict__ native, int64_t* __restrict__ win,
                                    int64_t* __restrict__ seq, int32_t* __restrict__ real, int batch, int k, int L,
                                    int hyb_min, int real_batch) {
  shk::pdl_trigger();
  shk::pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  if (b >= real_batch) {
    for (int j = 0; j <= k; ++j) win[(int64_t)b * (k + 1) + j] = 0;
    seq[b] = 0;
    real[b] = 0;
    return;
  }
  const int o = accept[b] + 1;
  const int64_t* c = cand + (int64_t)b * L;
  const int64_t* ot = out_tokens + (int64_t)b * (k + 1);
  const int cl = clen[b];
  bool aligned = o <= cl;
  for (int j = 0; j < o && aligned; ++j) aligned = c[j] == ot[j];
  int n_real = 0;
  if (aligned)
    while (n_real < k && o + n_real < cl) ++n_real;
  int64_t* w = win + (int64_t)b * (k + 1);
  w[0] = next_token[b];
  const bool use_native = native != nullptr && n_real < hyb_min;
  for (int j = 0; j < k; ++j)
    w[1 + j] = use_native ? native[(int64_t)b * k + j] : (j < n_real ? c[o + j] : -1);
  seq[b] = seq_new[b];
  real[b] = use_native ? 0 : n_real;
}

}  // namespace shk

using namespace shk;

void spec_advance(torch::Tensor out_tokens, torch::Tensor accept, torch::Tensor next_token, torch::Tensor seq_new,
                  torch::Tensor cand, torch::Tensor clen, c10::optional<torch::Tensor> native, torch::Tensor win,
                  torch::Tensor seq, torch::Tensor real, int64_t hyb_min, int64_t real_batch) {
  TORCH_CHECK(out_tokens.scalar_type() == at::kLong && cand.scalar_type() == at::kLong && win.scalar_type() == at::kLong &&
                  seq.scalar_type() == at::kLong && seq_new.scalar_type() == at::kLong &&
                  next_token.scalar_type() == at::kLong, "spec_advance: int64 tokens");
  TORCH_CHECK(accept.scalar_type() == at::kInt && clen.scalar_type() == at::kInt && real.scalar_type() == at::kInt,
              "spec_advance: int32 counts");
  TORCH_CHECK(out_tokens.is_contiguous() && cand.is_contiguous() && win.is_contiguous(), "spec_advance: contiguous");
  const int batch = win.size(0), k = win.size(1) - 1, L = cand.size(1);
  TORCH_CHECK(out_tokens.size(0) >= batch && out_tokens.size(1) == k + 1 && cand.size(0) >= batch,
              "spec_advance: shapes");
  const int64_t* nat = nullptr;
  if (native.has_value()) {
    TORCH_CHECK(native->scalar_type() == at::kLong && native->is_contiguous() && native->size(1) == k,
                "spec_advance: native [B, k]");
    nat = native->data_ptr<int64_t>();
  }
  if (batch == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  shk::launch(spec_advance_kernel, dim3((batch + 127) / 128), dim3(128), 0, stream, out_tokens.data_ptr<int64_t>(),
              accept.data_ptr<int32_t>(), next_token.data_ptr<int64_t>(), seq_new.data_ptr<int64_t>(),
              cand.data_ptr<int64_t>(), clen.data_ptr<int32_t>(), nat, win.data_ptr<int64_t>(),
              seq.data_ptr<int64_t>(), real.data_ptr<int32_t>(), batch, k, L, static_cast<int>(hyb_min),
              static_cast<int>(real_batch));
  SH_CUDA_CHECK(cudaGetLastError());
}

void argmax_rows(torch::Tensor out, torch::Tensor logits) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "argmax_rows: logits [T, V]");
  TORCH_CHECK(out.scalar_type() == at::kLong && out.numel() == logits.size(0), "argmax_rows: out int64 [T]");
  const int64_t rows = logits.size(0), vocab = logits.size(1);
  if (rows == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const bool aligned = (reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0) &&
                       (logits.stride(0) * logits.element_size()) % 16 == 0;
  TORCH_CHECK(aligned, "argmax_rows: logits rows must start on 16-byte boundaries");
  if (logits.scalar_type() == at::kBFloat16) {
    shk::launch(argmax_rows_kernel<__nv_bfloat16, 8>, dim3(rows), dim3(512), 0, stream, 
        out.data_ptr<int64_t>(), (const __nv_bfloat16*)logits.data_ptr(), vocab, logits.stride(0));
  } else if (logits.scalar_type() == at::kFloat) {
    shk::launch(argmax_rows_kernel<float, 4>, dim3(rows), dim3(512), 0, stream, out.data_ptr<int64_t>(), logits.data_ptr<float>(), vocab,
                                                           logits.stride(0));
  } else {
    TORCH_CHECK(false, "argmax_rows: bf16 or f32 logits");
  }
  SH_CUDA_CHECK(cudaGetLastError());
}

void spec_verify(torch::Tensor draft, torch::Tensor target, torch::Tensor seq_lens, torch::Tensor out_tokens,
                 torch::Tensor accept, torch::Tensor next_token) {
  TORCH_CHECK(draft.scalar_type() == at::kLong && target.scalar_type() == at::kLong, "spec_verify: int64 tokens");
  TORCH_CHECK(seq_lens.scalar_type() == at::kLong && accept.scalar_type() == at::kInt, "spec_verify: dtypes");
  TORCH_CHECK(draft.dim() == 2 && target.dim() == 2 && out_tokens.dim() == 2 && draft.stride(1) == 1 &&
                  target.stride(1) == 1 && out_tokens.stride(1) == 1, "spec_verify: row-major [B, *] views");
  const int batch = draft.size(0), k = draft.size(1);
  TORCH_CHECK(target.size(0) == batch && target.size(1) == k + 1, "target must be [B, k+1]");
  TORCH_CHECK(out_tokens.size(0) >= batch && out_tokens.size(1) == k + 1, "out_tokens must be [B, k+1]");
  if (batch == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  shk::launch(spec_verify_kernel, dim3((batch + 127) / 128), dim3(128), 0, stream, 
      draft.data_ptr<int64_t>(), target.data_ptr<int64_t>(), seq_lens.data_ptr<int64_t>(),
      out_tokens.data_ptr<int64_t>(), accept.data_ptr<int32_t>(), next_token.data_ptr<int64_t>(), batch, k,
      draft.stride(0), target.stride(0), out_tokens.stride(0));
  SH_CUDA_CHECK(cudaGetLastError());
}
