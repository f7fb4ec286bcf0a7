// Python bindings of the sm_100a kernel library (module `_C`).
#include <torch/extension.h>

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
}
