// Python bindings of the sm_100a kernel library (module `_C`).
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "gemm_tcgen05.h"

void rms_norm(torch::Tensor out, torch::Tensor x, torch::Tensor w, double eps);
void fused_add_rms_norm(torch::Tensor x, torch::Tensor residual, torch::Tensor w, double eps);
void rope_kv_write(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin, torch::Tensor k_cache,
                   torch::Tensor v_cache, torch::Tensor slot_mapping, int64_t hq, int64_t hk, int64_t d, int64_t rot);
void silu_mul(torch::Tensor out, torch::Tensor x);
void embedding(torch::Tensor out, torch::Tensor ids, torch::Tensor table);
void argmax_rows(torch::Tensor out, torch::Tensor logits);
void spec_verify(torch::Tensor draft, torch::Tensor target, torch::Tensor seq_lens, torch::Tensor out_tokens,
                 torch::Tensor accept, torch::Tensor next_token);
void paged_attention(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                     torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor q_start,
                     torch::Tensor tile_req, torch::Tensor tile_row0, int64_t hq, double scale);

// y[M, N] = x[M, K] @ w[N, K]^T via the tcgen05 GEMM.  swap: weights take the
// MMA's 128-row side (small M).  ws: fp32 split-K workspace (>= splits*M*N).
void gemm_bf16(torch::Tensor y, torch::Tensor x, torch::Tensor w, bool swap, int64_t bn, int64_t splits,
               c10::optional<torch::Tensor> ws, c10::optional<torch::Tensor> err) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && y.is_cuda(), "gemm_bf16: CUDA tensors");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16,
              "gemm_bf16: bf16 tensors");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 && y.stride(1) == 1,
              "gemm_bf16: row-major 2-D operands");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && y.size(0) == M && y.size(1) == N, "gemm_bf16: shape mismatch");
  static int num_sms = 0;
  if (!num_sms) num_sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  float* wsp = nullptr;
  if (ws.has_value()) {
    TORCH_CHECK(ws->scalar_type() == at::kFloat && ws->numel() >= splits * M * N, "gemm_bf16: workspace too small");
    wsp = ws->data_ptr<float>();
  }
  int* errp = err.has_value() ? err->data_ptr<int>() : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream();
  int r;
  if (swap)
    r = sh_gemm_bf16_tcgen05(w.data_ptr(), N, w.stride(0), x.data_ptr(), M, x.stride(0), K, y.data_ptr(), y.stride(0),
                             1, bn, splits, wsp, errp, num_sms, stream);
  else
    r = sh_gemm_bf16_tcgen05(x.data_ptr(), M, x.stride(0), w.data_ptr(), N, w.stride(0), K, y.data_ptr(), y.stride(0),
                             0, bn, splits, wsp, errp, num_sms, stream);
  TORCH_CHECK(r == 0, "sh_gemm_bf16_tcgen05 failed with code ", r);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 (sm_100a) kernels: fused norms, RoPE+cache write, paged attention, GEMMs, verify, comm";
  m.def("rms_norm", &rms_norm);
  m.def("fused_add_rms_norm", &fused_add_rms_norm);
  m.def("rope_kv_write", &rope_kv_write);
  m.def("silu_mul", &silu_mul);
  m.def("embedding", &embedding);
  m.def("argmax_rows", &argmax_rows);
  m.def("spec_verify", &spec_verify);
  m.def("paged_attention", &paged_attention);
  m.def("gemm_bf16", &gemm_bf16, "tcgen05 GEMM", py::arg("y"), py::arg("x"), py::arg("w"), py::arg("swap"),
        py::arg("bn"), py::arg("splits"), py::arg("ws") = py::none(), py::arg("err") = py::none());
}
