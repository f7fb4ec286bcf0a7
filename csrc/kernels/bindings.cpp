// Python bindings of the sm_100a kernel library (module `_C`).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAFunctions.h>
#include <cstring>
#include <torch/extension.h>

#include "gemm_tcgen05.h"
#include "comm.h"
#include "ep_a2a.h"
#include "gdn.h"
#include "moe.h"
#include "mla.h"
#include "hisparse.h"
#include "dsa_indexer.h"
#include "gemm_fp4mma.h"
#include "gemm_nvfp4.h"
#include "paged_attention.h"

void rms_norm(torch::Tensor out, torch::Tensor x, torch::Tensor w, double eps);
void fused_add_rms_norm(torch::Tensor x, torch::Tensor residual, torch::Tensor w, double eps);
void rope_kv_write(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin, torch::Tensor k_cache,
                   torch::Tensor v_cache, torch::Tensor slot_mapping, int64_t hq, int64_t hk, int64_t d, int64_t rot);
void silu_mul(torch::Tensor out, torch::Tensor x);
void embedding(torch::Tensor out, torch::Tensor ids, torch::Tensor table);
void argmax_rows(torch::Tensor out, torch::Tensor logits);
void spec_verify(torch::Tensor draft, torch::Tensor target, torch::Tensor seq_lens, torch::Tensor out_tokens,
                 torch::Tensor accept, torch::Tensor next_token);
void spec_advance(torch::Tensor out_tokens, torch::Tensor accept, torch::Tensor next_token, torch::Tensor seq_new,
                  torch::Tensor cand, torch::Tensor clen, c10::optional<torch::Tensor> native, torch::Tensor win,
                  torch::Tensor seq, torch::Tensor real, int64_t hyb_min, int64_t real_batch);

// out[T, hq*D] <- paged GQA attention of the q rows (a view into the QKV
// projection output) over the [blocks, hk, 64, D] cache.  nsplit > 1 needs
// part_o [T*hq*nsplit*D] and part_ml [T*hq*nsplit*2] fp32 workspaces.
void paged_attention(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                     torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor q_start,
                     torch::Tensor tile_req, torch::Tensor tile_row0, int64_t hq, double scale, int64_t nsplit,
                     c10::optional<torch::Tensor> part_o, c10::optional<torch::Tensor> part_ml,
                     c10::optional<torch::Tensor> err, int64_t max_rows) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k_cache.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16, "paged_attention: bf16 tensors");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == 64 && k_cache.is_contiguous() && v_cache.is_contiguous() &&
                  v_cache.sizes() == k_cache.sizes(), "paged_attention: caches [blocks, hk, 64, D] contiguous");
  TORCH_CHECK(q.stride(-1) == 1 && out.stride(-1) == 1 && q.dim() == 2 && out.dim() == 2, "q/out [T, width]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kLong &&
                  q_start.scalar_type() == at::kLong && tile_req.scalar_type() == at::kInt &&
                  tile_row0.scalar_type() == at::kInt, "paged_attention: index dtypes");
  const int hk = k_cache.size(1), d = k_cache.size(3);
  TORCH_CHECK(hq % hk == 0 && q.size(1) >= hq * d && out.size(1) >= hq * d, "paged_attention: head layout");
  TORCH_CHECK((q.stride(0) * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(q.data_ptr()) % 16) == 0,
              "paged_attention: q rows must be 16-byte aligned");
  AttnParams p{};
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.out_stride = out.stride(0);
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.q_stride = q.stride(0);
  p.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  p.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  p.block_tables = block_tables.data_ptr<int32_t>();
  p.bt_stride = block_tables.stride(0);
  p.seq_lens = seq_lens.data_ptr<int64_t>();
  p.q_start = q_start.data_ptr<int64_t>();
  p.tile_req = tile_req.data_ptr<int32_t>();
  p.tile_row0 = tile_row0.data_ptr<int32_t>();
  p.num_tokens = q.size(0);
  p.hq = static_cast<int>(hq);
  p.hk = hk;
  p.nsplit = static_cast<int>(nsplit);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  if (nsplit > 1) {
    TORCH_CHECK(part_o.has_value() && part_ml.has_value(), "paged_attention: split-KV needs workspaces");
    TORCH_CHECK(part_o->numel() >= p.num_tokens * hq * nsplit * d && part_ml->numel() >= p.num_tokens * hq * nsplit * 2,
                "paged_attention: workspace too small");
    p.part_o = part_o->data_ptr<float>();
    p.part_ml = part_ml->data_ptr<float>();
  }
  p.err = err.has_value() ? err->data_ptr<int>() : nullptr;
  TORCH_CHECK(max_rows >= 1 && max_rows <= 64, "paged_attention: max_rows in 1..64");
  const int r = sh_paged_attention(&p, static_cast<int>(tile_req.numel()), static_cast<int>(k_cache.size(0)), d,
                                   static_cast<int>(max_rows), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_paged_attention failed with code ", r);
}

// y[M, N] = x[M, K] @ w[N, K]^T via the tcgen05 GEMM.  swap: weights take the
// MMA's 128-row side (small M).  ws: fp32 split-K workspace (>= splits*M*N).
void gemm_bf16(torch::Tensor y, torch::Tensor x, torch::Tensor w, bool swap, int64_t bn, int64_t splits,
               c10::optional<torch::Tensor> ws, c10::optional<torch::Tensor> err, bool pair) {
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
  auto fn = pair ? sh_gemm_bf16_pair : sh_gemm_bf16_tcgen05;
  int r;
  if (swap)
    r = fn(w.data_ptr(), N, w.stride(0), x.data_ptr(), M, x.stride(0), K, y.data_ptr(), y.stride(0), 1, bn, splits, wsp,
           errp, num_sms, stream);
  else
    r = fn(x.data_ptr(), M, x.stride(0), w.data_ptr(), N, w.stride(0), K, y.data_ptr(), y.stride(0), 0, bn, splits, wsp,
           errp, num_sms, stream);
  TORCH_CHECK(r == 0, pair ? "sh_gemm_bf16_pair" : "sh_gemm_bf16_tcgen05", " failed with code ", r);
}

// Limit of every cross-rank wait of the comm and EP kernels launched from here
// (ns; 0 = each kernel's default of 5 s).  set_wait_ns changes it for the
// process: serving keeps the default, tests shorten it to make a wait run out.
static unsigned long long g_wait_ns = 0;
void set_wait_ns(int64_t ns) { g_wait_ns = ns > 0 ? static_cast<unsigned long long>(ns) : 0ull; }
int64_t get_wait_ns() { return static_cast<int64_t>(g_wait_ns); }

// y[M, N] = x[M, K] @ w[N, K]^T via the stream-K CTA-pair kernel (weights on
// the MMA M side, ns*nsub tokens per tile).  ws / cnt: see sh_gemm_bf16_sk.
void gemm_bf16_sk(torch::Tensor y, torch::Tensor x, torch::Tensor w, int64_t ns, int64_t nsub, int64_t clusters,
                  torch::Tensor ws, torch::Tensor cnt, c10::optional<torch::Tensor> err,
                  c10::optional<torch::Tensor> stamps) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && y.is_cuda() && ws.is_cuda() && cnt.is_cuda(), "gemm_bf16_sk: CUDA tensors");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16,
              "gemm_bf16_sk: bf16 tensors");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && y.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 && y.stride(1) == 1,
              "gemm_bf16_sk: row-major 2-D operands");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && y.size(0) == M && y.size(1) == N, "gemm_bf16_sk: shape mismatch");
  int64_t tiles = 0, need = 0;
  TORCH_CHECK(sh_gemm_sk_shape(static_cast<int>(N), static_cast<int>(M), static_cast<int>(K), static_cast<int>(ns),
                               static_cast<int>(nsub), static_cast<int>(clusters), &tiles, &need) == 0,
              "gemm_bf16_sk: bad shape");
  TORCH_CHECK(ws.scalar_type() == at::kFloat && ws.numel() >= need, "gemm_bf16_sk: workspace too small");
  TORCH_CHECK(cnt.scalar_type() == at::kInt && cnt.numel() >= 2 * tiles, "gemm_bf16_sk: counter array too small");
  int* errp = err.has_value() ? err->data_ptr<int>() : nullptr;
  unsigned long long* st = nullptr;
  if (stamps.has_value()) {
    TORCH_CHECK(stamps->scalar_type() == at::kLong && stamps->is_cuda() && stamps->numel() >= 2 * clusters * 64,
                "gemm_bf16_sk: stamps int64 [2 * clusters, 64]");
    st = reinterpret_cast<unsigned long long*>(stamps->data_ptr<int64_t>());
  }
  const int r = sh_gemm_bf16_sk(w.data_ptr(), static_cast<int>(N), w.stride(0), x.data_ptr(), static_cast<int>(M),
                                x.stride(0), static_cast<int>(K), y.data_ptr(), y.stride(0), static_cast<int>(ns),
                                static_cast<int>(nsub), static_cast<int>(clusters), ws.data_ptr<float>(),
                                cnt.data_ptr<int>(), errp, st, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_gemm_bf16_sk failed with code ", r);
}

int64_t gemm_sk_max_clusters(int64_t ns, int64_t nsub) {
  return sh_gemm_sk_max_clusters(static_cast<int>(ns), static_cast<int>(nsub));
}

// Vocab-parallel greedy argmax over NVLink peer memory (one kernel; see ArgmaxParams).
void argmax_tp(torch::Tensor out, torch::Tensor logits, std::vector<int64_t> peer_keys,
               std::vector<int64_t> peer_flags, torch::Tensor counters, torch::Tensor err, int64_t rank,
               int64_t max_T, int64_t vocab_offset, int64_t num_blocks) {
  const int world = static_cast<int>(peer_keys.size());
  TORCH_CHECK(world >= 1 && world <= SH_COMM_MAX_WORLD && peer_flags.size() == peer_keys.size(), "argmax_tp: peers");
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1,
              "argmax_tp: bf16 logits [T, V_local]");
  TORCH_CHECK(out.scalar_type() == at::kLong && out.is_contiguous() && out.numel() == logits.size(0), "argmax_tp: out");
  TORCH_CHECK(counters.scalar_type() == at::kInt && counters.numel() >= SH_COMM_MAX_BLOCKS, "argmax_tp: counters");
  ArgmaxParams p{};
  p.logits = reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr());
  p.ld = logits.stride(0);
  for (int i = 0; i < world; ++i) {
    p.peer_keys[i] = reinterpret_cast<unsigned long long*>(peer_keys[i]);
    p.peer_flags[i] = reinterpret_cast<uint32_t*>(peer_flags[i]);
  }
  p.counters = reinterpret_cast<uint32_t*>(counters.data_ptr<int>());
  p.out = out.data_ptr<int64_t>();
  p.err = err.data_ptr<int>();
  p.rank = static_cast<int>(rank);
  p.world = world;
  p.T = static_cast<int>(logits.size(0));
  p.V_local = static_cast<int>(logits.size(1));
  p.max_T = static_cast<int>(max_T);
  p.vocab_offset = vocab_offset;
  p.wait_ns = g_wait_ns;
  const int r = sh_argmax_tp(&p, static_cast<int>(num_blocks), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_argmax_tp failed with code ", r);
}

// Fused NVLink all-reduce (+ residual add + RMSNorm).  peer_* are device
// addresses (ints) of every rank's symmetric receive / gather buffers and
// flag arrays; `partial` is this rank's [T, H] partial in local memory.
void allreduce_fused(torch::Tensor partial, std::vector<int64_t> peer_recv, std::vector<int64_t> peer_gather,
                     std::vector<int64_t> peer_flags, torch::Tensor counters, torch::Tensor out,
                     c10::optional<torch::Tensor> residual, c10::optional<torch::Tensor> weight, torch::Tensor err,
                     int64_t rank, int64_t T, int64_t H, int64_t max_T, double eps, bool two_shot,
                     int64_t num_blocks, c10::optional<torch::Tensor> timing, int64_t prefetch_ptr,
                     int64_t prefetch_bytes, int64_t quant) {
  const int world = static_cast<int>(peer_recv.size());
  TORCH_CHECK(world >= 1 && world <= SH_COMM_MAX_WORLD && peer_gather.size() == peer_recv.size() &&
                  peer_flags.size() == peer_recv.size(), "allreduce_fused: peer lists");
  TORCH_CHECK(partial.is_cuda() && partial.scalar_type() == at::kBFloat16 && partial.is_contiguous() &&
                  partial.numel() >= T * H, "allreduce_fused: partial");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() >= T * H, "out");
  TORCH_CHECK(counters.scalar_type() == at::kInt && counters.numel() >= SH_COMM_MAX_BLOCKS, "counters");
  TORCH_CHECK(T <= max_T, "allreduce_fused: T exceeds the receive slots");
  ArParams p{};
  p.partial = reinterpret_cast<const __nv_bfloat16*>(partial.data_ptr());
  for (int i = 0; i < world; ++i) {
    p.peer_recv[i] = reinterpret_cast<__nv_bfloat16*>(peer_recv[i]);
    p.peer_gather[i] = reinterpret_cast<__nv_bfloat16*>(peer_gather[i]);
    p.peer_flags[i] = reinterpret_cast<uint32_t*>(peer_flags[i]);
  }
  p.counters = reinterpret_cast<uint32_t*>(counters.data_ptr<int>());
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.fuse_norm = residual.has_value() ? 1 : 0;
  if (p.fuse_norm) {
    TORCH_CHECK(weight.has_value() && residual->is_contiguous() && residual->scalar_type() == at::kBFloat16,
                "allreduce_fused: residual/weight");
    p.residual = reinterpret_cast<__nv_bfloat16*>(residual->data_ptr());
    p.weight = reinterpret_cast<const __nv_bfloat16*>(weight->data_ptr());
  }
  p.err = err.data_ptr<int>();
  p.rank = static_cast<int>(rank);
  p.world = world;
  p.T = static_cast<int>(T);
  p.H = static_cast<int>(H);
  p.max_T = static_cast<int>(max_T);
  p.eps = static_cast<float>(eps);
  p.two_shot = two_shot ? 1 : 0;
  if (timing.has_value()) {
    TORCH_CHECK(timing->scalar_type() == at::kLong && timing->numel() >= 256, "allreduce_fused: timing [64, 4] int64");
    p.timing = reinterpret_cast<unsigned long long*>(timing->data_ptr<int64_t>());
  }
  p.prefetch = reinterpret_cast<const void*>(prefetch_ptr);
  p.prefetch_bytes = static_cast<unsigned long long>(prefetch_bytes > 0 ? prefetch_bytes : 0);
  p.wait_ns = g_wait_ns;
  p.quant = static_cast<int>(quant);
  const int r = sh_allreduce(&p, static_cast<int>(num_blocks), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_allreduce failed with code ", r);
}

// Row-parallel GEMM y = x w^T whose epilogue pushes output rows to their owner
// ranks' receive slots (reduce-scatter inside the GEMM), see GemmParams::push.
void gemm_bf16_push(torch::Tensor x, torch::Tensor w, bool pair, int64_t bn, std::vector<int64_t> peer_recv,
                    std::vector<int64_t> peer_cnt, torch::Tensor counters, int64_t rank, int64_t push_rows,
                    int64_t max_T, c10::optional<torch::Tensor> err) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "gemm_bf16_push: bf16 CUDA tensors");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1, "gemm_bf16_push: 2-D row-major");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && M <= max_T, "gemm_bf16_push: shapes");
  const int world = static_cast<int>(peer_recv.size());
  TORCH_CHECK(world >= 1 && world <= 8 && peer_cnt.size() == peer_recv.size(), "gemm_bf16_push: peer lists");
  TORCH_CHECK(counters.scalar_type() == at::kInt, "gemm_bf16_push: counters");
  static int num_sms = 0;
  if (!num_sms) num_sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  GemmParams g{};
  for (int i = 0; i < world; ++i) {
    g.push_recv[i] = reinterpret_cast<__nv_bfloat16*>(peer_recv[i]);
    g.push_cnt[i] = reinterpret_cast<uint32_t*>(peer_cnt[i]);
  }
  g.push_epoch = reinterpret_cast<const uint32_t*>(counters.data_ptr<int>());
  g.push_rank = static_cast<int>(rank);
  g.push_world = world;
  g.push_rows = static_cast<int>(push_rows);
  g.push_max_T = static_cast<int>(max_T);
  g.push_n = static_cast<int>(N);
  int* errp = err.has_value() ? err->data_ptr<int>() : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int r = sh_gemm_bf16_push(x.data_ptr(), M, x.stride(0), w.data_ptr(), N, w.stride(0), K, 0, bn, pair ? 1 : 0,
                                  &g, errp, num_sms, stream);
  TORCH_CHECK(r == 0, "sh_gemm_bf16_push failed with code ", r);
}

void rs_norm_ag(int64_t recv, std::vector<int64_t> peer_gather, std::vector<int64_t> peer_gather_res,
                std::vector<int64_t> peer_flags, int64_t rs_cnt, torch::Tensor targets, torch::Tensor counters,
                torch::Tensor residual, torch::Tensor out, torch::Tensor weight, torch::Tensor err, int64_t rank,
                int64_t T, int64_t H, int64_t max_T, int64_t Tc, int64_t expected, double eps, bool gather_res,
                int64_t num_blocks, c10::optional<torch::Tensor> timing, int64_t prefetch_ptr,
                int64_t prefetch_bytes) {
  const int world = static_cast<int>(peer_gather.size());
  TORCH_CHECK(world >= 1 && world <= SH_COMM_MAX_WORLD && peer_flags.size() == peer_gather.size() &&
                  peer_gather_res.size() == peer_gather.size(), "rs_norm_ag: peer lists");
  TORCH_CHECK(residual.scalar_type() == at::kBFloat16 && residual.is_contiguous() && residual.numel() >= T * H &&
                  out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() >= T * H &&
                  weight.scalar_type() == at::kBFloat16 && weight.numel() == H, "rs_norm_ag: tensors");
  TORCH_CHECK(targets.scalar_type() == at::kInt && targets.numel() >= 2 * SH_COMM_MAX_BLOCKS &&
                  counters.scalar_type() == at::kInt && counters.numel() >= SH_COMM_MAX_BLOCKS, "rs_norm_ag: state");
  RsParams p{};
  p.recv = reinterpret_cast<const __nv_bfloat16*>(recv);
  for (int i = 0; i < world; ++i) {
    p.peer_gather[i] = reinterpret_cast<__nv_bfloat16*>(peer_gather[i]);
    p.peer_gather_res[i] = reinterpret_cast<__nv_bfloat16*>(peer_gather_res[i]);
    p.peer_flags[i] = reinterpret_cast<uint32_t*>(peer_flags[i]);
  }
  p.rs_cnt = reinterpret_cast<uint32_t*>(rs_cnt);
  p.targets = reinterpret_cast<uint32_t*>(targets.data_ptr<int>());
  p.counters = reinterpret_cast<uint32_t*>(counters.data_ptr<int>());
  p.residual = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.weight = reinterpret_cast<const __nv_bfloat16*>(weight.data_ptr());
  p.err = err.data_ptr<int>();
  p.rank = static_cast<int>(rank);
  p.world = world;
  p.T = static_cast<int>(T);
  p.H = static_cast<int>(H);
  p.max_T = static_cast<int>(max_T);
  p.Tc = static_cast<int>(Tc);
  p.expected = static_cast<uint32_t>(expected);
  p.eps = static_cast<float>(eps);
  p.gather_res = gather_res ? 1 : 0;
  if (timing.has_value()) p.timing = reinterpret_cast<unsigned long long*>(timing->data_ptr<int64_t>());
  p.prefetch = reinterpret_cast<const void*>(prefetch_ptr);
  p.prefetch_bytes = static_cast<unsigned long long>(prefetch_bytes > 0 ? prefetch_bytes : 0);
  p.wait_ns = g_wait_ns;
  const int r = sh_rs_norm_ag(&p, static_cast<int>(num_blocks), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_rs_norm_ag failed with code ", r);
}

// --- MLA decode / DSA indexer -----------------------------------------------------
void mla_decode(torch::Tensor out, torch::Tensor q, torch::Tensor latent, torch::Tensor block_tables,
                torch::Tensor seq_lens, torch::Tensor q_start, c10::optional<torch::Tensor> topk, int64_t nsplit,
                c10::optional<torch::Tensor> part_o, c10::optional<torch::Tensor> part_ml, double scale,
                torch::Tensor err, int64_t impl, c10::optional<torch::Tensor> stamps) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.is_contiguous(), "mla: q [T,H,C]");
  const bool fp4 = latent.scalar_type() == at::kByte;
  TORCH_CHECK((fp4 || latent.scalar_type() == at::kBFloat16) && latent.dim() == 3 && latent.size(1) == 64 &&
                  latent.is_contiguous(), "mla: latent [blocks, 64, C] bf16 or NVFP4 rows [blocks, 64, row_bytes]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.dim() == 3, "mla: out [T,H,V]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kLong &&
                  q_start.scalar_type() == at::kLong, "mla: index dtypes");
  const int C = static_cast<int>(q.size(2)), V = static_cast<int>(out.size(2));
  TORCH_CHECK(latent.size(2) == (fp4 ? sh_mla_fp4_row_bytes(V, C - V) : C), "mla: latent width");
  MlaParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  if (fp4)
    p.latent_fp4 = latent.data_ptr<uint8_t>();
  else
    p.latent = reinterpret_cast<const __nv_bfloat16*>(latent.data_ptr());
  p.block_tables = block_tables.data_ptr<int32_t>();
  p.bt_stride = block_tables.stride(0);
  p.seq_lens = seq_lens.data_ptr<int64_t>();
  p.q_start = q_start.data_ptr<int64_t>();
  p.B = static_cast<int>(seq_lens.size(0));
  if (topk.has_value()) {
    TORCH_CHECK(topk->scalar_type() == at::kInt && topk->is_contiguous() && topk->size(0) == q.size(0), "mla: topk");
    p.topk = topk->data_ptr<int32_t>();
    p.topk_k = static_cast<int>(topk->size(1));
  }
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.nsplit = static_cast<int>(nsplit);
  if (nsplit > 1) {
    TORCH_CHECK(part_o.has_value() && part_ml.has_value() && part_o->numel() >= q.size(0) * q.size(1) * nsplit * V &&
                    part_ml->numel() >= q.size(0) * q.size(1) * nsplit * 2, "mla: split workspace");
    p.part_o = part_o->data_ptr<float>();
    p.part_ml = part_ml->data_ptr<float>();
  }
  p.err = err.data_ptr<int>();
  p.T = static_cast<int>(q.size(0));
  p.H = static_cast<int>(q.size(1));
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.impl = static_cast<int>(impl);
  if (stamps) {
    TORCH_CHECK(stamps->scalar_type() == at::kLong && stamps->is_cuda(), "mla: stamps int64");
    p.stamps = reinterpret_cast<unsigned long long*>(stamps->data_ptr<int64_t>());
  }
  const int r = sh_mla_decode(&p, C, V, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_mla_decode failed with code ", r, " (C=", C, ", V=", V, ")");
}

// Pinned host memory mapped into the device address space, as a CUDA uint8 tensor over the device-side
// pointer: kernels read and write it over the host link (zero-copy).  Zero-filled; freed with the tensor.
torch::Tensor mapped_host_buffer(int64_t nbytes) {
  TORCH_CHECK(nbytes > 0, "mapped_host_buffer: size");
  void* h = nullptr;
  cudaError_t e = cudaHostAlloc(&h, static_cast<size_t>(nbytes), cudaHostAllocMapped | cudaHostAllocPortable);
  TORCH_CHECK(e == cudaSuccess, "cudaHostAlloc(", nbytes, " bytes) failed: ", cudaGetErrorString(e));
  void* d = nullptr;
  e = cudaHostGetDevicePointer(&d, h, 0);
  if (e != cudaSuccess) {
    cudaFreeHost(h);
    TORCH_CHECK(false, "cudaHostGetDevicePointer failed: ", cudaGetErrorString(e));
  }
  std::memset(h, 0, static_cast<size_t>(nbytes));
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, c10::cuda::current_device());
  return torch::from_blob(d, {nbytes}, [h](void*) { cudaFreeHost(h); }, opts);
}

void hisparse_resolve(torch::Tensor topk, torch::Tensor topk_out, torch::Tensor q_start, torch::Tensor seq_lens,
                      torch::Tensor state_slots, torch::Tensor positions, torch::Tensor slot_mapping,
                      torch::Tensor block_tables, torch::Tensor cold, torch::Tensor hot, torch::Tensor pos2slot,
                      torch::Tensor slot2pos, torch::Tensor stamp, torch::Tensor clock, torch::Tensor hot_bt,
                      torch::Tensor hot_seq, torch::Tensor err, c10::optional<torch::Tensor> stats) {
  const int64_t B = seq_lens.size(0), T = topk.size(0);
  TORCH_CHECK(topk.scalar_type() == at::kInt && topk_out.scalar_type() == at::kInt && topk.is_contiguous() &&
                  topk_out.is_contiguous() && topk_out.size(0) >= T && topk_out.size(1) == topk.size(1),
              "hisparse: top-k lists int32 [T, K]");
  TORCH_CHECK(q_start.scalar_type() == at::kLong && seq_lens.scalar_type() == at::kLong &&
                  state_slots.scalar_type() == at::kLong && positions.scalar_type() == at::kLong &&
                  slot_mapping.scalar_type() == at::kLong && q_start.size(0) == B + 1 && state_slots.size(0) >= B &&
                  positions.size(0) >= T && slot_mapping.size(0) >= T,
              "hisparse: int64 batch metadata");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.stride(1) == 1 && block_tables.size(0) >= B,
              "hisparse: block tables int32");
  const int64_t row_bytes = cold.numel() / (cold.size(0) * cold.size(1)) * cold.element_size();
  TORCH_CHECK(cold.is_contiguous() && hot.is_contiguous() && cold.size(1) == 64 && hot.size(1) == 64 &&
                  cold.scalar_type() == hot.scalar_type() && hot.numel() * hot.element_size() % row_bytes == 0 &&
                  hot.numel() / (hot.size(0) * hot.size(1)) * hot.element_size() == row_bytes,
              "hisparse: cold and hot caches [blocks, 64, row] of one row format");
  TORCH_CHECK(pos2slot.scalar_type() == at::kInt && slot2pos.scalar_type() == at::kInt &&
                  stamp.scalar_type() == at::kInt && clock.scalar_type() == at::kInt && pos2slot.is_contiguous() &&
                  slot2pos.is_contiguous() && stamp.is_contiguous() && pos2slot.dim() == 2 && slot2pos.dim() == 2 &&
                  stamp.sizes() == slot2pos.sizes() && clock.size(0) == slot2pos.size(0) &&
                  pos2slot.size(0) == slot2pos.size(0),
              "hisparse: residency maps int32 [slots, P], [slots, H]");
  const int64_t H = slot2pos.size(1);
  TORCH_CHECK(hot.size(0) * 64 >= slot2pos.size(0) * H, "hisparse: hot rows < slots x H");
  TORCH_CHECK(hot_bt.scalar_type() == at::kInt && hot_bt.is_contiguous() && hot_bt.numel() >= B * (H / 64) &&
                  hot_seq.scalar_type() == at::kLong && hot_seq.size(0) >= B && err.scalar_type() == at::kInt,
              "hisparse: outputs");
  HsParams p{};
  p.topk = topk.data_ptr<int32_t>();
  p.topk_out = topk_out.data_ptr<int32_t>();
  p.q_start = q_start.data_ptr<int64_t>();
  p.seq_lens = seq_lens.data_ptr<int64_t>();
  p.state_slots = state_slots.data_ptr<int64_t>();
  p.positions = positions.data_ptr<int64_t>();
  p.slot_mapping = slot_mapping.data_ptr<int64_t>();
  p.block_tables = block_tables.data_ptr<int32_t>();
  p.bt_stride = block_tables.stride(0);
  p.cold = reinterpret_cast<const uint8_t*>(cold.data_ptr());
  p.hot = reinterpret_cast<uint8_t*>(hot.data_ptr());
  p.pos2slot = pos2slot.data_ptr<int32_t>();
  p.slot2pos = slot2pos.data_ptr<int32_t>();
  p.stamp = stamp.data_ptr<int32_t>();
  p.clock = clock.data_ptr<int32_t>();
  p.hot_bt = hot_bt.data_ptr<int32_t>();
  p.hot_seq = hot_seq.data_ptr<int64_t>();
  p.err = err.data_ptr<int>();
  if (stats) {
    TORCH_CHECK(stats->scalar_type() == at::kLong && stats->numel() >= 2, "hisparse: stats int64 [2]");
    p.stats = stats->data_ptr<int64_t>();
  }
  p.B = static_cast<int>(B);
  p.K = static_cast<int>(topk.size(1));
  p.H = static_cast<int>(H);
  p.P = static_cast<int>(pos2slot.size(1));
  p.row_bytes = static_cast<int>(row_bytes);
  const int r = sh_hisparse_resolve(&p, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_hisparse_resolve failed with code ", r);
}

void hisparse_reset(torch::Tensor pos2slot, torch::Tensor slot2pos, torch::Tensor stamp, torch::Tensor clock,
                    torch::Tensor slots) {
  TORCH_CHECK(pos2slot.dim() == 3 && slot2pos.dim() == 3 && pos2slot.is_contiguous() && slot2pos.is_contiguous() &&
                  stamp.is_contiguous() && clock.is_contiguous() && stamp.sizes() == slot2pos.sizes() &&
                  clock.size(0) == pos2slot.size(0) && clock.size(1) == pos2slot.size(1) &&
                  slots.scalar_type() == at::kLong && pos2slot.scalar_type() == at::kInt,
              "hisparse_reset: maps [layers, slots, P] / [layers, slots, H] int32, slots int64");
  const int r = sh_hisparse_reset(pos2slot.data_ptr<int32_t>(), slot2pos.data_ptr<int32_t>(), stamp.data_ptr<int32_t>(),
                                  clock.data_ptr<int32_t>(), slots.data_ptr<int64_t>(), static_cast<int>(slots.numel()),
                                  static_cast<int>(pos2slot.size(0)), static_cast<int>(pos2slot.size(1)),
                                  static_cast<int>(slot2pos.size(2)), static_cast<int>(pos2slot.size(2)),
                                  at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_hisparse_reset failed with code ", r);
}

void mla_cache_write(torch::Tensor latent, torch::Tensor c, torch::Tensor kpe, torch::Tensor slots) {
  if (latent.scalar_type() == at::kByte) {  // NVFP4 latent rows
    TORCH_CHECK(c.scalar_type() == at::kBFloat16 && kpe.scalar_type() == at::kBFloat16 &&
                    slots.scalar_type() == at::kLong && c.stride(1) == 1 && kpe.stride(1) == 1 &&
                    latent.is_contiguous() && latent.size(2) == sh_mla_fp4_row_bytes(c.size(1), kpe.size(1)),
                "mla_cache_write: NVFP4 cache rows");
    const int r = sh_mla_cache_write_fp4(latent.data_ptr<uint8_t>(), reinterpret_cast<const __nv_bfloat16*>(c.data_ptr()),
                                         c.stride(0), reinterpret_cast<const __nv_bfloat16*>(kpe.data_ptr()),
                                         kpe.stride(0), slots.data_ptr<int64_t>(), static_cast<int>(c.size(0)),
                                         static_cast<int>(c.size(1)), static_cast<int>(kpe.size(1)),
                                         at::cuda::getCurrentCUDAStream());
    TORCH_CHECK(r == 0, "sh_mla_cache_write_fp4 failed with code ", r);
    return;
  }
  TORCH_CHECK(latent.scalar_type() == at::kBFloat16 && c.scalar_type() == at::kBFloat16 &&
                  kpe.scalar_type() == at::kBFloat16 && slots.scalar_type() == at::kLong, "mla_cache_write: dtypes");
  TORCH_CHECK(c.stride(1) == 1 && kpe.stride(1) == 1 && latent.size(2) == c.size(1) + kpe.size(1), "mla_cache_write");
  const int r = sh_mla_cache_write(reinterpret_cast<__nv_bfloat16*>(latent.data_ptr()),
                                   reinterpret_cast<const __nv_bfloat16*>(c.data_ptr()), c.stride(0),
                                   reinterpret_cast<const __nv_bfloat16*>(kpe.data_ptr()), kpe.stride(0),
                                   slots.data_ptr<int64_t>(), static_cast<int>(c.size(0)), static_cast<int>(c.size(1)),
                                   static_cast<int>(kpe.size(1)), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_mla_cache_write failed with code ", r);
}

// Indexer key cache: page [64 x 128 e4m3 | 64 f32 scales] (8448 bytes) per 64 slots.
void dsa_cache_write(torch::Tensor cache, torch::Tensor k, torch::Tensor slots) {
  TORCH_CHECK(cache.scalar_type() == at::kByte && cache.dim() == 2 && cache.size(1) == SH_DSA_PAGE_BYTES &&
                  cache.is_contiguous() && cache.is_cuda(),
              "dsa_cache_write: cache [pages, 8448] uint8");
  TORCH_CHECK(k.scalar_type() == at::kBFloat16 && k.dim() == 2 && k.size(1) == SH_DSA_DIM && k.stride(1) == 1,
              "dsa_cache_write: k [T, 128] bf16 with unit inner stride");
  TORCH_CHECK(slots.scalar_type() == at::kLong && slots.is_contiguous() && slots.numel() == k.size(0),
              "dsa_cache_write: slots [T] int64");
  const int r = sh_dsa_cache_write(cache.data_ptr<uint8_t>(), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()),
                                   k.stride(0), slots.data_ptr<int64_t>(), static_cast<int>(k.size(0)),
                                   at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_dsa_cache_write failed with code ", r);
}

// q8 = e4m3 queries, wq = w * per-row query scale (rows of 128 values).
void dsa_quant_q(torch::Tensor q8, torch::Tensor wq, torch::Tensor q, torch::Tensor w) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.size(2) == SH_DSA_DIM && q.is_contiguous(),
              "dsa_quant_q: q [T, IH, 128] bf16 contiguous");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.numel() == q.size(0) * q.size(1),
              "dsa_quant_q: w [T, IH] fp32");
  TORCH_CHECK(q8.scalar_type() == at::kByte && q8.is_contiguous() && q8.numel() == q.numel(), "dsa_quant_q: q8");
  TORCH_CHECK(wq.scalar_type() == at::kFloat && wq.is_contiguous() && wq.numel() == w.numel(), "dsa_quant_q: wq");
  const int r = sh_dsa_quant_q(q8.data_ptr<uint8_t>(), wq.data_ptr<float>(),
                               reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), w.data_ptr<float>(),
                               static_cast<int>(w.numel()), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_dsa_quant_q failed with code ", r);
}

// Indexer logits into `logits` rows and (unless score_only) the top-K positions per query row.
void dsa_index(torch::Tensor topk, torch::Tensor logits, torch::Tensor q8, torch::Tensor wq, torch::Tensor cache,
               torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor q_start, int64_t grid,
               c10::optional<torch::Tensor> err, bool score_only) {
  TORCH_CHECK(q8.scalar_type() == at::kByte && q8.dim() == 3 && q8.size(2) == SH_DSA_DIM && q8.is_contiguous(),
              "dsa_index: q8 [T, IH, 128] uint8");
  TORCH_CHECK(wq.scalar_type() == at::kFloat && wq.is_contiguous() && wq.numel() == q8.size(0) * q8.size(1),
              "dsa_index: wq [T, IH] fp32");
  TORCH_CHECK(cache.scalar_type() == at::kByte && cache.dim() == 2 && cache.size(1) == SH_DSA_PAGE_BYTES &&
                  cache.is_contiguous(),
              "dsa_index: cache [pages, 8448] uint8");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1 &&
                  logits.size(0) >= q8.size(0) && logits.stride(0) % 4 == 0 &&
                  logits.size(1) >= block_tables.size(1) * SH_DSA_PAGE_KEYS,
              "dsa_index: logits [T, >= max_keys] fp32 rows (row stride a multiple of 4)");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.dim() == 2 && block_tables.stride(1) == 1,
              "dsa_index: block_tables int32 [B, W]");
  TORCH_CHECK(seq_lens.scalar_type() == at::kLong && q_start.scalar_type() == at::kLong &&
                  q_start.numel() == seq_lens.numel() + 1 && block_tables.size(0) >= seq_lens.numel(),
              "dsa_index: seq_lens [B], q_start [B + 1] int64");
  if (!score_only)
    TORCH_CHECK(topk.scalar_type() == at::kInt && topk.dim() == 2 && topk.is_contiguous() &&
                    topk.size(0) == q8.size(0),
                "dsa_index: topk [T, K] int32");
  if (err) TORCH_CHECK(err->scalar_type() == at::kInt && err->numel() >= 1, "dsa_index: err int32");
  DsaIndexParams p{};
  p.q8 = q8.data_ptr<uint8_t>();
  p.wq = wq.data_ptr<float>();
  p.kcache = cache.data_ptr<uint8_t>();
  p.num_pages = static_cast<int>(cache.size(0));
  p.block_tables = block_tables.data_ptr<int32_t>();
  p.bt_stride = block_tables.stride(0);
  p.seq_lens = seq_lens.data_ptr<int64_t>();
  p.q_start = q_start.data_ptr<int64_t>();
  p.B = static_cast<int>(seq_lens.numel());
  p.T = static_cast<int>(q8.size(0));
  p.IH = static_cast<int>(q8.size(1));
  p.K = score_only ? 0 : static_cast<int>(topk.size(1));
  p.logits = logits.data_ptr<float>();
  p.ld = logits.stride(0);
  p.topk = score_only ? nullptr : topk.data_ptr<int32_t>();
  p.err = err ? err->data_ptr<int>() : nullptr;
  p.grid = static_cast<int>(grid);
  const int r = score_only ? sh_dsa_score(&p, at::cuda::getCurrentCUDAStream())
                           : sh_dsa_index(&p, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_dsa_index failed with code ", r, " (IH=", p.IH, ")");
}

// NVFP4-weight GEMM (W4A16): y[t, n] = x[t] . dequant(W[n]); grouped MoE mode with `groups`.
void gemm_nvfp4(torch::Tensor y, torch::Tensor x, torch::Tensor packed, torch::Tensor scales, torch::Tensor gscale,
                int64_t bn, c10::optional<torch::Tensor> groups, c10::optional<torch::Tensor> num_groups,
                int64_t rows_p, c10::optional<torch::Tensor> err, int64_t splits, c10::optional<torch::Tensor> ws) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "gemm_nvfp4: x");
  TORCH_CHECK(packed.scalar_type() == at::kByte && packed.is_contiguous() && scales.is_contiguous() &&
                  scales.element_size() == 1 && gscale.scalar_type() == at::kFloat, "gemm_nvfp4: weights");
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.stride(1) == 1, "gemm_nvfp4: y");
  const int64_t K = x.size(1);
  // scales: k-block-major [K/64, rows_pad, 4] (see ops.nvfp4_kmajor_scales)
  TORCH_CHECK(packed.size(1) * 2 == K && scales.dim() == 3 && scales.size(0) * 64 == K && scales.size(2) == 4 &&
                  scales.size(1) >= packed.size(0) && scales.size(1) % 128 == 0, "gemm_nvfp4: shapes");
  static int num_sms = 0;
  if (!num_sms) num_sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  Fp4GemmParams g{};
  g.packed = packed.data_ptr<uint8_t>();
  g.scales = reinterpret_cast<const uint8_t*>(scales.data_ptr());
  g.global_scale = gscale.data_ptr<float>();
  g.out = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  g.ldo = y.stride(0);
  g.rows_total = static_cast<int>(packed.size(0));
  g.rows_pad = static_cast<int>(scales.size(1));
  g.K = static_cast<int>(K);
  g.err = err.has_value() ? err->data_ptr<int>() : nullptr;
  if (groups.has_value()) {
    TORCH_CHECK(num_groups.has_value() && groups->scalar_type() == at::kInt && groups->size(1) == 4, "gemm_nvfp4: groups");
    g.groups = reinterpret_cast<const int4*>(groups->data_ptr<int>());
    g.num_groups = num_groups->data_ptr<int>();
    g.max_groups = static_cast<int>(groups->size(0));
    g.rows_p = static_cast<int>(rows_p);
  }
  if (splits > 1) {
    TORCH_CHECK(ws.has_value() && ws->scalar_type() == at::kFloat && ws->numel() >= splits * x.size(0) * packed.size(0),
                "gemm_nvfp4: split workspace");
    g.ws = ws->data_ptr<float>();
  }
  const int r = sh_gemm_nvfp4(&g, x.data_ptr(), static_cast<int>(x.size(0)), x.stride(0), static_cast<int>(bn),
                              static_cast<int>(splits), num_sms, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_gemm_nvfp4 failed with code ", r);
}

// NVFP4 activation quantiser (see sh_nvfp4_quant_act): x bf16 [rows, K] ->
// xq uint8 [rows, K/2], x_sf uint8 [tiles, kc4, 512], a_scale fp32 [rows].
void nvfp4_gather_act(torch::Tensor codes, torch::Tensor scales, torch::Tensor ascale, torch::Tensor token,
                      torch::Tensor groups, torch::Tensor num_groups, torch::Tensor xq, torch::Tensor x_sf,
                      torch::Tensor a_scale) {
  TORCH_CHECK(codes.is_cuda() && codes.scalar_type() == at::kByte && codes.is_contiguous() && codes.dim() == 2,
              "nvfp4_gather_act: codes uint8 [rows, K/2]");
  const int64_t K = codes.size(1) * 2, rows = token.numel();
  TORCH_CHECK(scales.scalar_type() == at::kByte && scales.is_contiguous() && scales.size(1) * 16 == K &&
                  scales.size(0) == codes.size(0), "nvfp4_gather_act: scales uint8 [rows, K/16]");
  TORCH_CHECK(ascale.scalar_type() == at::kFloat && ascale.numel() >= codes.size(0), "nvfp4_gather_act: ascale");
  TORCH_CHECK(token.scalar_type() == at::kInt && token.is_contiguous(), "nvfp4_gather_act: token int32");
  TORCH_CHECK(groups.scalar_type() == at::kInt && groups.size(1) == 4 && num_groups.scalar_type() == at::kInt,
              "nvfp4_gather_act: groups");
  TORCH_CHECK(xq.scalar_type() == at::kByte && xq.is_contiguous() && xq.size(0) >= rows && xq.size(1) * 2 == K,
              "nvfp4_gather_act: xq uint8 [pairs, K/2]");
  const int64_t kc4 = (K + 255) / 256 * 4;
  TORCH_CHECK(x_sf.element_size() == 1 && x_sf.is_contiguous() && x_sf.size(1) == kc4 && x_sf.size(2) == 512 &&
                  x_sf.size(0) >= groups.size(0), "nvfp4_gather_act: x_sf [tiles, kc4, 512]");
  TORCH_CHECK(a_scale.scalar_type() == at::kFloat && a_scale.numel() >= rows, "nvfp4_gather_act: a_scale");
  const int r = sh_nvfp4_gather_act(codes.data_ptr<uint8_t>(), scales.data_ptr<uint8_t>(), ascale.data_ptr<float>(),
                                    token.data_ptr<int>(), static_cast<int>(rows), static_cast<int>(K),
                                    reinterpret_cast<const int4*>(groups.data_ptr<int>()), num_groups.data_ptr<int>(),
                                    xq.data_ptr<uint8_t>(), reinterpret_cast<uint8_t*>(x_sf.data_ptr()),
                                    a_scale.data_ptr<float>(), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_nvfp4_gather_act failed with code ", r);
}

void nvfp4_quant_act(torch::Tensor x, torch::Tensor xq, torch::Tensor x_sf, torch::Tensor a_scale, int64_t tile_rows,
                     double static_g, c10::optional<torch::Tensor> groups, c10::optional<torch::Tensor> num_groups,
                     bool swiglu) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "nvfp4_quant_act: x bf16 [rows, K] (or [rows, 2K] gate | up with swiglu)");
  TORCH_CHECK(!swiglu || x.size(1) % 2 == 0, "nvfp4_quant_act: swiglu needs an even width");
  const int64_t rows = x.size(0), K = swiglu ? x.size(1) / 2 : x.size(1);
  TORCH_CHECK(xq.scalar_type() == at::kByte && xq.is_contiguous() && xq.size(0) >= rows && xq.size(1) * 2 == K,
              "nvfp4_quant_act: xq uint8 [rows, K/2]");
  const int64_t kc4 = (K + 255) / 256 * 4;
  TORCH_CHECK(x_sf.element_size() == 1 && x_sf.is_contiguous() && x_sf.dim() == 3 && x_sf.size(1) == kc4 &&
                  x_sf.size(2) == 512, "nvfp4_quant_act: x_sf [tiles, kc4, 512]");
  TORCH_CHECK(a_scale.scalar_type() == at::kFloat && a_scale.numel() >= rows, "nvfp4_quant_act: a_scale");
  const int4* gp = nullptr;
  const int* ng = nullptr;
  int64_t max_tiles = (rows + tile_rows - 1) / tile_rows;
  if (groups.has_value()) {
    TORCH_CHECK(num_groups.has_value() && groups->scalar_type() == at::kInt && groups->size(1) == 4,
                "nvfp4_quant_act: groups");
    gp = reinterpret_cast<const int4*>(groups->data_ptr<int>());
    ng = num_groups->data_ptr<int>();
    max_tiles = groups->size(0);
  }
  TORCH_CHECK(x_sf.size(0) >= max_tiles, "nvfp4_quant_act: x_sf has too few tiles");
  const int r = sh_nvfp4_quant_act(x.data_ptr(), x.stride(0), static_cast<int>(rows), static_cast<int>(K), gp, ng,
                                   static_cast<int>(max_tiles), static_cast<int>(tile_rows),
                                   static_cast<float>(static_g), xq.data_ptr<uint8_t>(),
                                   reinterpret_cast<uint8_t*>(x_sf.data_ptr()), a_scale.data_ptr<float>(),
                                   swiglu ? 1 : 0, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_nvfp4_quant_act failed with code ", r);
}

// Block-scaled W4A4 GEMM (see sh_gemm_fp4mma): y[t, n] = alpha_w * a_scale[t] * (xq sx) . (w sw).
void gemm_fp4mma(torch::Tensor y, torch::Tensor xq, torch::Tensor x_sf, torch::Tensor a_scale, torch::Tensor w,
                 torch::Tensor w_sf, torch::Tensor alpha_w, int64_t bn, c10::optional<torch::Tensor> groups,
                 c10::optional<torch::Tensor> num_groups, int64_t rows_p, c10::optional<torch::Tensor> err,
                 int64_t splits, c10::optional<torch::Tensor> ws, c10::optional<torch::Tensor> counters,
                 bool fp8, c10::optional<torch::Tensor> stamps) {
  TORCH_CHECK(xq.is_cuda() && xq.scalar_type() == at::kByte && xq.is_contiguous() && xq.dim() == 2, "gemm_fp4mma: xq");
  TORCH_CHECK(w.scalar_type() == at::kByte && w.is_contiguous() && w.size(1) == xq.size(1), "gemm_fp4mma: w");
  // NVFP4: two codes per byte, 4 scale chunks per 256 k; MXFP8: one code per byte, one chunk per 128 k
  const int64_t K = fp8 ? xq.size(1) : xq.size(1) * 2, kc4 = fp8 ? K / 128 : (K + 255) / 256 * 4;
  TORCH_CHECK(w_sf.element_size() == 1 && w_sf.is_contiguous() && w_sf.dim() == 3 && w_sf.size(1) == kc4 &&
                  w_sf.size(2) == 512 && x_sf.element_size() == 1 && x_sf.is_contiguous() && x_sf.dim() == 3 &&
                  x_sf.size(1) == kc4, "gemm_fp4mma: scale tiles [tiles, kc4, 512]");
  TORCH_CHECK(alpha_w.scalar_type() == at::kFloat && a_scale.scalar_type() == at::kFloat &&
                  a_scale.numel() >= xq.size(0), "gemm_fp4mma: scales");
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.stride(1) == 1 && y.size(0) >= xq.size(0), "gemm_fp4mma: y");
  static int num_sms = 0;
  if (!num_sms) num_sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  Fp4MmaParams g{};
  g.w = w.data_ptr<uint8_t>();
  g.w_sf = reinterpret_cast<const uint8_t*>(w_sf.data_ptr());
  g.alpha_w = alpha_w.data_ptr<float>();
  g.x_sf = reinterpret_cast<const uint8_t*>(x_sf.data_ptr());
  g.a_scale = a_scale.data_ptr<float>();
  g.out = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  g.ldo = y.stride(0);
  g.rows_total = static_cast<int>(w.size(0));
  g.K = static_cast<int>(K);
  g.err = err.has_value() ? err->data_ptr<int>() : nullptr;
  const int64_t rows_m = groups.has_value() ? rows_p : w.size(0);
  TORCH_CHECK(w_sf.size(0) >= (groups.has_value() ? (w.size(0) / rows_p) : 1) * ((rows_m + 127) / 128),
              "gemm_fp4mma: w_sf has too few tiles");
  if (groups.has_value()) {
    TORCH_CHECK(num_groups.has_value() && groups->scalar_type() == at::kInt && groups->size(1) == 4 && rows_p > 0 &&
                    w.size(0) % rows_p == 0, "gemm_fp4mma: groups");
    TORCH_CHECK(x_sf.size(0) >= groups->size(0), "gemm_fp4mma: one activation scale tile per group entry");
    g.groups = reinterpret_cast<const int4*>(groups->data_ptr<int>());
    g.num_groups = num_groups->data_ptr<int>();
    g.max_groups = static_cast<int>(groups->size(0));
    g.rows_p = static_cast<int>(rows_p);
  } else {
    TORCH_CHECK(x_sf.size(0) >= (xq.size(0) + bn - 1) / bn, "gemm_fp4mma: activation scale tiles of bn rows");
  }
  if (splits > 1 && !groups.has_value()) {
    const int64_t tiles = ((w.size(0) + 127) / 128) * ((xq.size(0) + bn - 1) / bn);
    TORCH_CHECK(ws.has_value() && ws->scalar_type() == at::kFloat && ws->numel() >= splits * tiles * 128 * bn,
                "gemm_fp4mma: split workspace of splits * tiles * 128 * bn floats");
    TORCH_CHECK(counters.has_value() && counters->scalar_type() == at::kInt && counters->numel() >= tiles,
                "gemm_fp4mma: split tickets (zeroed int32 per output tile)");
    g.ws = ws->data_ptr<float>();
    g.counters = counters->data_ptr<int>();
  }
  if (stamps) {
    TORCH_CHECK(stamps->scalar_type() == at::kLong && stamps->is_cuda() && stamps->numel() >= 8 * num_sms,
                "gemm_fp4mma: stamps int64 [num_sms * 8]");
    g.stamps = reinterpret_cast<unsigned long long*>(stamps->data_ptr<int64_t>());
  }
  const int r = (fp8 ? sh_gemm_mxfp8 : sh_gemm_fp4mma)(&g, xq.data_ptr(), static_cast<int>(xq.size(0)),
                                                       static_cast<int>(bn), static_cast<int>(splits), num_sms,
                                                       at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "block-scaled GEMM failed with code ", r);
}

// MXFP8 activation quantiser (see sh_mxfp8_quant_act): x bf16 [rows, K] -> xq [rows, K] e4m3,
// x_sf [tiles, K/128, 512] ue8m0, a_scale [rows] = 1.
void mxfp8_quant_act(torch::Tensor x, torch::Tensor xq, torch::Tensor x_sf, torch::Tensor a_scale, int64_t tile_rows,
                     c10::optional<torch::Tensor> groups, c10::optional<torch::Tensor> num_groups) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "mxfp8: x");
  const int64_t rows = x.size(0), K = x.size(1);
  TORCH_CHECK(xq.scalar_type() == at::kByte && xq.is_contiguous() && xq.size(0) >= rows && xq.size(1) == K,
              "mxfp8: xq uint8 [rows, K]");
  TORCH_CHECK(x_sf.element_size() == 1 && x_sf.is_contiguous() && x_sf.dim() == 3 && x_sf.size(1) == K / 128 &&
                  x_sf.size(2) == 512, "mxfp8: x_sf [tiles, K/128, 512]");
  TORCH_CHECK(a_scale.scalar_type() == at::kFloat && a_scale.numel() >= rows, "mxfp8: a_scale");
  const int4* gp = nullptr;
  const int* ng = nullptr;
  int64_t tiles = (rows + tile_rows - 1) / tile_rows;
  if (groups.has_value()) {
    TORCH_CHECK(num_groups.has_value() && groups->scalar_type() == at::kInt, "mxfp8: groups");
    gp = reinterpret_cast<const int4*>(groups->data_ptr<int>());
    ng = num_groups->data_ptr<int>();
    tiles = groups->size(0);
  }
  TORCH_CHECK(x_sf.size(0) >= tiles, "mxfp8: x_sf has too few tiles");
  const int r = sh_mxfp8_quant_act(x.data_ptr(), x.stride(0), static_cast<int>(rows), static_cast<int>(K), gp, ng,
                                   static_cast<int>(tile_rows), xq.data_ptr<uint8_t>(),
                                   reinterpret_cast<uint8_t*>(x_sf.data_ptr()), a_scale.data_ptr<float>(),
                                   at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(r == 0, "sh_mxfp8_quant_act failed with code ", r);
}

template <typename T>
static T* ptr(const torch::Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}
#define SH_CHECK_RC(rc, what) TORCH_CHECK((rc) == 0, what " failed with code ", (rc))

// --- Gated DeltaNet -----------------------------------------------------------
void gdn_conv(torch::Tensor x, torch::Tensor w, torch::Tensor y, torch::Tensor state, torch::Tensor rec_x,
              torch::Tensor pending, torch::Tensor slots, torch::Tensor q_start, int64_t W, int64_t mode) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kFloat &&
                  state.scalar_type() == at::kFloat && rec_x.scalar_type() == at::kFloat, "gdn_conv dtypes");
  GdnConvParams p{};
  p.x = ptr<const __nv_bfloat16>(x);
  p.x_stride = x.stride(0);
  p.w = ptr<const float>(w);
  p.y = ptr<__nv_bfloat16>(y);
  p.state = ptr<float>(state);
  p.rec_x = ptr<float>(rec_x);
  p.pending = ptr<const int32_t>(pending);
  p.slots = ptr<const int64_t>(slots);
  p.q_start = ptr<const int64_t>(q_start);
  p.C = static_cast<int>(w.size(0));
  p.KW = static_cast<int>(w.size(1));
  p.W = static_cast<int>(W);
  p.mode = static_cast<int>(mode);
  SH_CHECK_RC(sh_gdn_conv(&p, static_cast<int>(slots.numel()), at::cuda::getCurrentCUDAStream()), "sh_gdn_conv");
}

void gdn_recurrent(torch::Tensor qkv, torch::Tensor z, torch::Tensor ba, torch::Tensor a_log, torch::Tensor dt_bias,
                   torch::Tensor norm_w, torch::Tensor state, torch::Tensor rec_k, torch::Tensor rec_v,
                   torch::Tensor rec_g, torch::Tensor rec_b, torch::Tensor pending, torch::Tensor slots,
                   torch::Tensor q_start, torch::Tensor out, int64_t H, int64_t HV, int64_t K, int64_t W,
                   int64_t mode, double eps) {
  TORCH_CHECK(state.scalar_type() == at::kFloat && qkv.scalar_type() == at::kBFloat16, "gdn_recurrent dtypes");
  GdnParams p{};
  p.qkv = ptr<const __nv_bfloat16>(qkv);
  p.qkv_stride = qkv.stride(0);
  p.z = ptr<const __nv_bfloat16>(z);
  p.z_stride = z.stride(0);
  p.ba = ptr<const __nv_bfloat16>(ba);
  p.ba_stride = ba.stride(0);
  p.a_log = ptr<const float>(a_log);
  p.dt_bias = ptr<const float>(dt_bias);
  p.norm_w = ptr<const __nv_bfloat16>(norm_w);
  p.state = ptr<float>(state);
  p.rec_k = ptr<float>(rec_k);
  p.rec_v = ptr<float>(rec_v);
  p.rec_g = ptr<float>(rec_g);
  p.rec_b = ptr<float>(rec_b);
  p.pending = ptr<const int32_t>(pending);
  p.slots = ptr<const int64_t>(slots);
  p.q_start = ptr<const int64_t>(q_start);
  p.out = ptr<__nv_bfloat16>(out);
  p.out_stride = out.stride(0);
  p.H = static_cast<int>(H);
  p.HV = static_cast<int>(HV);
  p.K = static_cast<int>(K);
  p.V = static_cast<int>(K);
  p.W = static_cast<int>(W);
  p.mode = static_cast<int>(mode);
  p.eps = static_cast<float>(eps);
  SH_CHECK_RC(sh_gdn_recurrent(&p, static_cast<int>(slots.numel()), at::cuda::getCurrentCUDAStream()),
              "sh_gdn_recurrent");
}

// --- expert-parallel all-to-all over NVLink peer memory ------------------------
static EpParams ep_params(torch::Tensor ids, std::vector<int64_t> peer_x, std::vector<int64_t> peer_ids,
                          std::vector<int64_t> peer_w, std::vector<int64_t> peer_y, std::vector<int64_t> peer_flags,
                          torch::Tensor counters, torch::Tensor err, int64_t rank, int64_t H, int64_t e_local,
                          int64_t max_T) {
  const int world = static_cast<int>(peer_x.size());
  TORCH_CHECK(world >= 1 && world <= SH_EP_MAX_WORLD && peer_ids.size() == peer_x.size() &&
                  peer_w.size() == peer_x.size() && peer_y.size() == peer_x.size() &&
                  peer_flags.size() == peer_x.size(), "ep: peer lists");
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kInt && ids.is_contiguous() && ids.dim() == 2, "ep: ids");
  TORCH_CHECK(counters.scalar_type() == at::kInt && counters.numel() >= SH_EP_MAX_BLOCKS, "ep: counters");
  TORCH_CHECK(ids.size(0) <= max_T, "ep: T exceeds the receive buffers");
  EpParams p{};
  p.ids = ids.data_ptr<int32_t>();
  for (int i = 0; i < world; ++i) {
    p.peer_x[i] = reinterpret_cast<__nv_bfloat16*>(peer_x[i]);
    p.peer_ids[i] = reinterpret_cast<int32_t*>(peer_ids[i]);
    p.peer_w[i] = reinterpret_cast<float*>(peer_w[i]);
    p.peer_y[i] = reinterpret_cast<__nv_bfloat16*>(peer_y[i]);
    p.peer_flags[i] = reinterpret_cast<uint32_t*>(peer_flags[i]);
  }
  p.counters = reinterpret_cast<uint32_t*>(counters.data_ptr<int>());
  p.err = err.data_ptr<int>();
  p.rank = static_cast<int>(rank);
  p.world = world;
  p.T = static_cast<int>(ids.size(0));
  p.k = static_cast<int>(ids.size(1));
  p.H = static_cast<int>(H);
  p.e_local = static_cast<int>(e_local);
  p.max_T = static_cast<int>(max_T);
  p.wait_ns = g_wait_ns;
  return p;
}

void ep_dispatch(torch::Tensor x, torch::Tensor ids, torch::Tensor w, std::vector<int64_t> peer_x,
                 std::vector<int64_t> peer_ids, std::vector<int64_t> peer_w, std::vector<int64_t> peer_y,
                 std::vector<int64_t> peer_flags, torch::Tensor counters, torch::Tensor err, int64_t rank,
                 int64_t e_local, int64_t max_T, int64_t num_blocks, std::vector<int64_t> peer_q,
                 std::vector<int64_t> peer_s, std::vector<int64_t> peer_a, c10::optional<torch::Tensor> logits,
                 c10::optional<torch::Tensor> bias, bool sigmoid_grouped, int64_t n_groups, int64_t topk_groups,
                 bool renorm, double scale) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.size(0) == ids.size(0),
              "ep_dispatch: x");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.sizes() == ids.sizes(), "ep_dispatch: w");
  EpParams p = ep_params(ids, peer_x, peer_ids, peer_w, peer_y, peer_flags, counters, err, rank, x.size(1), e_local,
                         max_T);
  p.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  p.w = w.data_ptr<float>();
  if (logits.has_value()) {  // the dispatch routes its tokens; ids / w are written, not read
    TORCH_CHECK(logits->is_cuda() && logits->is_contiguous() && logits->dim() == 2 &&
                    logits->size(0) == ids.size(0) &&
                    (logits->scalar_type() == at::kFloat || logits->scalar_type() == at::kBFloat16),
                "ep_dispatch: logits fp32/bf16 [T, E]");
    RouteParams& r = p.route;
    r.logits = logits->data_ptr();
    r.logits_bf16 = logits->scalar_type() == at::kBFloat16 ? 1 : 0;
    if (bias.has_value()) {
      TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == logits->size(1), "ep_dispatch: bias");
      r.bias = bias->data_ptr<float>();
    }
    r.ids = ids.data_ptr<int32_t>();
    r.weights = w.data_ptr<float>();
    r.T = static_cast<int>(ids.size(0));
    r.E = static_cast<int>(logits->size(1));
    r.k = static_cast<int>(ids.size(1));
    r.sigmoid_grouped = sigmoid_grouped ? 1 : 0;
    r.n_groups = static_cast<int>(n_groups);
    r.topk_groups = static_cast<int>(topk_groups);
    r.renorm = renorm ? 1 : 0;
    r.scale = static_cast<float>(scale);
    p.fused_route = 1;
  }
  if (!peer_q.empty()) {  // NVFP4 dispatch
    TORCH_CHECK(peer_q.size() == peer_x.size() && peer_s.size() == peer_x.size() && peer_a.size() == peer_x.size(),
                "ep_dispatch: quantised peer lists");
    p.quant = 1;
    for (size_t i = 0; i < peer_q.size(); ++i) {
      p.peer_q[i] = reinterpret_cast<uint8_t*>(peer_q[i]);
      p.peer_s[i] = reinterpret_cast<uint8_t*>(peer_s[i]);
      p.peer_a[i] = reinterpret_cast<float*>(peer_a[i]);
    }
  }
  SH_CHECK_RC(sh_ep_dispatch(&p, static_cast<int>(num_blocks), at::cuda::getCurrentCUDAStream()), "sh_ep_dispatch");
}

void ep_combine(torch::Tensor y, torch::Tensor ids, torch::Tensor out, std::vector<int64_t> peer_x,
                std::vector<int64_t> peer_ids, std::vector<int64_t> peer_w, std::vector<int64_t> peer_y,
                std::vector<int64_t> peer_flags, torch::Tensor counters, torch::Tensor err, int64_t rank,
                int64_t e_local, int64_t max_T, int64_t num_blocks) {
  const int64_t world = static_cast<int64_t>(peer_x.size());
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.is_contiguous() &&
                  y.size(0) == world * ids.size(0), "ep_combine: y [world*T, H]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.size(0) == ids.size(0) &&
                  out.size(1) == y.size(1), "ep_combine: out");
  EpParams p = ep_params(ids, peer_x, peer_ids, peer_w, peer_y, peer_flags, counters, err, rank, y.size(1), e_local,
                         max_T);
  p.y = reinterpret_cast<const __nv_bfloat16*>(y.data_ptr());
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  SH_CHECK_RC(sh_ep_combine(&p, static_cast<int>(num_blocks), at::cuda::getCurrentCUDAStream()), "sh_ep_combine");
}

void gdn_chunk_prefill(torch::Tensor qkv, torch::Tensor z, torch::Tensor ba, torch::Tensor a_log, torch::Tensor dt_bias,
                       torch::Tensor norm_w, torch::Tensor state, torch::Tensor slots, torch::Tensor q_start,
                       torch::Tensor out, int64_t H, int64_t HV, int64_t K, double eps, c10::optional<torch::Tensor> err) {
  TORCH_CHECK(state.scalar_type() == at::kFloat && qkv.scalar_type() == at::kBFloat16, "gdn_chunk_prefill dtypes");
  GdnParams p{};
  p.qkv = ptr<const __nv_bfloat16>(qkv);
  p.qkv_stride = qkv.stride(0);
  p.z = ptr<const __nv_bfloat16>(z);
  p.z_stride = z.stride(0);
  p.ba = ptr<const __nv_bfloat16>(ba);
  p.ba_stride = ba.stride(0);
  p.a_log = ptr<const float>(a_log);
  p.dt_bias = ptr<const float>(dt_bias);
  p.norm_w = ptr<const __nv_bfloat16>(norm_w);
  p.state = ptr<float>(state);
  p.slots = ptr<const int64_t>(slots);
  p.q_start = ptr<const int64_t>(q_start);
  p.out = ptr<__nv_bfloat16>(out);
  p.out_stride = out.stride(0);
  p.H = static_cast<int>(H);
  p.HV = static_cast<int>(HV);
  p.K = static_cast<int>(K);
  p.V = static_cast<int>(K);
  p.eps = static_cast<float>(eps);
  p.err = err.has_value() ? ptr<int32_t>(*err) : nullptr;
  SH_CHECK_RC(sh_gdn_chunk_prefill(&p, static_cast<int>(slots.numel()), at::cuda::getCurrentCUDAStream()),
              "sh_gdn_chunk_prefill");
}

void ep_combine_push(torch::Tensor ys, torch::Tensor sorted_pos, torch::Tensor w_local, torch::Tensor ids_local,
                     int64_t T, std::vector<int64_t> peer_x, std::vector<int64_t> peer_ids, std::vector<int64_t> peer_w,
                     std::vector<int64_t> peer_y, std::vector<int64_t> peer_flags, torch::Tensor counters,
                     torch::Tensor err, int64_t rank, int64_t e_local, int64_t max_T, int64_t num_blocks) {
  const int64_t world = static_cast<int64_t>(peer_x.size());
  TORCH_CHECK(ys.is_cuda() && ys.scalar_type() == at::kBFloat16 && ys.is_contiguous() && ys.dim() == 2,
              "ep_combine_push: ys bf16 [pairs, H]");
  TORCH_CHECK(ids_local.scalar_type() == at::kInt && ids_local.dim() == 2 && ids_local.size(0) == world * T,
              "ep_combine_push: ids_local [world*T, k]");
  TORCH_CHECK(sorted_pos.scalar_type() == at::kInt && sorted_pos.is_contiguous() &&
                  sorted_pos.numel() == ids_local.numel(), "ep_combine_push: sorted_pos [world*T*k]");
  TORCH_CHECK(w_local.scalar_type() == at::kFloat && w_local.is_contiguous() && w_local.numel() == ids_local.numel(),
              "ep_combine_push: w_local [world*T, k]");
  // ids of T tokens only give T and k here; the kernel reads the received local ids from peer_ids[rank].
  torch::Tensor shape_ids = ids_local.narrow(0, 0, T);
  EpParams p = ep_params(shape_ids.contiguous(), peer_x, peer_ids, peer_w, peer_y, peer_flags, counters, err, rank,
                         ys.size(1), e_local, max_T);
  p.ys = reinterpret_cast<const __nv_bfloat16*>(ys.data_ptr());
  p.sorted_pos = sorted_pos.data_ptr<int32_t>();
  p.w_local = w_local.data_ptr<float>();
  SH_CHECK_RC(sh_ep_combine_push(&p, static_cast<int>(num_blocks), at::cuda::getCurrentCUDAStream()),
              "sh_ep_combine_push");
}

void ep_combine_sum(torch::Tensor ids, torch::Tensor out, std::vector<int64_t> peer_x, std::vector<int64_t> peer_ids,
                    std::vector<int64_t> peer_w, std::vector<int64_t> peer_y, std::vector<int64_t> peer_flags,
                    torch::Tensor counters, torch::Tensor err, int64_t rank, int64_t e_local, int64_t max_T,
                    int64_t num_blocks) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.size(0) == ids.size(0),
              "ep_combine_sum: out [T, H]");
  EpParams p = ep_params(ids, peer_x, peer_ids, peer_w, peer_y, peer_flags, counters, err, rank, out.size(1), e_local,
                         max_T);
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.pushed = 1;
  SH_CHECK_RC(sh_ep_combine(&p, static_cast<int>(num_blocks), at::cuda::getCurrentCUDAStream()), "sh_ep_combine");
}

// --- MoE -------------------------------------------------------------------------
void moe_route(torch::Tensor logits, c10::optional<torch::Tensor> bias, torch::Tensor ids, torch::Tensor weights,
               int64_t k, bool sigmoid_grouped, int64_t n_groups, int64_t topk_groups, bool renorm, double scale) {
  RouteParams p{};
  p.logits = logits.data_ptr();
  p.logits_bf16 = logits.scalar_type() == at::kBFloat16;
  TORCH_CHECK(p.logits_bf16 || logits.scalar_type() == at::kFloat, "router logits bf16/f32");
  p.bias = bias.has_value() ? ptr<const float>(*bias) : nullptr;
  p.ids = ptr<int32_t>(ids);
  p.weights = ptr<float>(weights);
  p.T = static_cast<int>(logits.size(0));
  p.E = static_cast<int>(logits.size(1));
  p.k = static_cast<int>(k);
  p.sigmoid_grouped = sigmoid_grouped;
  p.n_groups = static_cast<int>(n_groups);
  p.topk_groups = static_cast<int>(topk_groups);
  p.renorm = renorm;
  p.scale = static_cast<float>(scale);
  SH_CHECK_RC(sh_moe_route(&p, at::cuda::getCurrentCUDAStream()), "sh_moe_route");
}

void moe_align(torch::Tensor ids, torch::Tensor rank, torch::Tensor offsets, torch::Tensor sorted_pos,
               torch::Tensor sorted_token, torch::Tensor groups, torch::Tensor num_groups, int64_t E, int64_t bn,
               int64_t rows_per_expert) {
  AlignParams p{};
  p.ids = ptr<const int32_t>(ids);
  p.rank = ptr<int32_t>(rank);
  p.offsets = ptr<int32_t>(offsets);
  p.sorted_pos = ptr<int32_t>(sorted_pos);
  p.sorted_token = ptr<int32_t>(sorted_token);
  p.groups = ptr<int4>(groups);
  p.num_groups = ptr<int>(num_groups);
  p.T = static_cast<int>(ids.size(0));
  p.k = static_cast<int>(ids.size(1));
  p.E = static_cast<int>(E);
  p.bn = static_cast<int>(bn);
  p.max_groups = static_cast<int>(groups.size(0));
  p.rows_per_expert = static_cast<int>(rows_per_expert);
  SH_CHECK_RC(sh_moe_align(&p, at::cuda::getCurrentCUDAStream()), "sh_moe_align");
}

void moe_gather(torch::Tensor out, torch::Tensor x, torch::Tensor sorted_token, torch::Tensor total) {
  SH_CHECK_RC(sh_moe_gather(ptr<__nv_bfloat16>(out), ptr<const __nv_bfloat16>(x), ptr<const int32_t>(sorted_token),
                            ptr<const int>(total), static_cast<int>(out.size(0)), static_cast<int>(x.size(1)),
                            at::cuda::getCurrentCUDAStream()),
              "sh_moe_gather");
}

void moe_combine(torch::Tensor out, torch::Tensor y, torch::Tensor sorted_pos, torch::Tensor w, bool accumulate) {
  SH_CHECK_RC(sh_moe_combine(ptr<__nv_bfloat16>(out), ptr<const __nv_bfloat16>(y), ptr<const int32_t>(sorted_pos),
                             ptr<const float>(w), static_cast<int>(out.size(0)), static_cast<int>(w.size(1)),
                             static_cast<int>(out.size(1)), accumulate, at::cuda::getCurrentCUDAStream()),
              "sh_moe_combine");
}

// Grouped expert GEMM: out[q_total, rows_p] over device-side tiles (see gemm_tcgen05.h).
void gemm_grouped(torch::Tensor out, torch::Tensor q, torch::Tensor w_stacked, int64_t rows_p, torch::Tensor groups,
                  torch::Tensor num_groups, int64_t bn) {
  static int num_sms = 0;
  if (!num_sms) num_sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  TORCH_CHECK(q.is_contiguous() && w_stacked.is_contiguous() && out.is_contiguous(), "gemm_grouped: contiguous");
  SH_CHECK_RC(sh_gemm_bf16_grouped(w_stacked.data_ptr(), static_cast<int>(w_stacked.size(0)), static_cast<int>(rows_p),
                                   q.data_ptr(), static_cast<int>(q.size(0)), static_cast<int>(q.size(1)),
                                   out.data_ptr(), out.stride(0), ptr<const int4>(groups), ptr<const int>(num_groups),
                                   static_cast<int>(groups.size(0)), static_cast<int>(bn), nullptr, num_sms,
                                   at::cuda::getCurrentCUDAStream()),
              "sh_gemm_bf16_grouped");
}

// --- NVFP4 ---------------------------------------------------------------------
extern "C" int sh_nvfp4_dequant(__nv_bfloat16* out, const uint8_t* packed, const uint8_t* scales, const float* global,
                                int64_t N, int K, cudaStream_t stream);
extern "C" int sh_nvfp4_quant(uint8_t* packed, uint8_t* scales, const __nv_bfloat16* w, const float* global, int64_t N,
                              int K, cudaStream_t stream);

void nvfp4_dequant(torch::Tensor out, torch::Tensor packed, torch::Tensor scales, torch::Tensor global) {
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && packed.is_contiguous() &&
                  scales.is_contiguous(), "nvfp4_dequant: contiguous bf16 out / uint8 packed / e4m3 scales");
  SH_CHECK_RC(sh_nvfp4_dequant(ptr<__nv_bfloat16>(out), ptr<const uint8_t>(packed), ptr<const uint8_t>(scales),
                               ptr<const float>(global), out.size(0), static_cast<int>(out.size(1)),
                               at::cuda::getCurrentCUDAStream()),
              "sh_nvfp4_dequant");
}

void nvfp4_quant(torch::Tensor packed, torch::Tensor scales, torch::Tensor w, torch::Tensor global) {
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous(), "nvfp4_quant: contiguous bf16 weight");
  SH_CHECK_RC(sh_nvfp4_quant(ptr<uint8_t>(packed), ptr<uint8_t>(scales), ptr<const __nv_bfloat16>(w),
                             ptr<const float>(global), w.size(0), static_cast<int>(w.size(1)),
                             at::cuda::getCurrentCUDAStream()),
              "sh_nvfp4_quant");
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
  m.def("paged_attention", &paged_attention, "paged GQA attention", py::arg("out"), py::arg("q"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("block_tables"), py::arg("seq_lens"), py::arg("q_start"), py::arg("tile_req"),
        py::arg("tile_row0"), py::arg("hq"), py::arg("scale"), py::arg("nsplit") = 1, py::arg("part_o") = py::none(),
        py::arg("part_ml") = py::none(), py::arg("err") = py::none(), py::arg("max_rows") = 64);
  m.def("allreduce_fused", &allreduce_fused, py::arg("partial"), py::arg("peer_recv"), py::arg("peer_gather"),
        py::arg("peer_flags"), py::arg("counters"), py::arg("out"), py::arg("residual"), py::arg("weight"),
        py::arg("err"), py::arg("rank"), py::arg("T"), py::arg("H"), py::arg("max_T"), py::arg("eps"),
        py::arg("two_shot"), py::arg("num_blocks"), py::arg("timing") = py::none(), py::arg("prefetch_ptr") = 0,
        py::arg("prefetch_bytes") = 0, py::arg("quant") = 0);
  m.def("gemm_bf16_push", &gemm_bf16_push);
  m.def("set_wait_ns", &set_wait_ns, "limit of every cross-rank wait of the comm / EP kernels (ns, 0 = 5 s)");
  m.def("get_wait_ns", &get_wait_ns);
  m.def("argmax_tp", &argmax_tp, "vocab-parallel greedy argmax over NVLink peer memory", py::arg("out"),
        py::arg("logits"), py::arg("peer_keys"), py::arg("peer_flags"), py::arg("counters"), py::arg("err"),
        py::arg("rank"), py::arg("max_T"), py::arg("vocab_offset"), py::arg("num_blocks"));
  m.def("rs_norm_ag", &rs_norm_ag, py::arg("recv"), py::arg("peer_gather"), py::arg("peer_gather_res"),
        py::arg("peer_flags"), py::arg("rs_cnt"), py::arg("targets"), py::arg("counters"), py::arg("residual"),
        py::arg("out"), py::arg("weight"), py::arg("err"), py::arg("rank"), py::arg("T"), py::arg("H"),
        py::arg("max_T"), py::arg("Tc"), py::arg("expected"), py::arg("eps"), py::arg("gather_res"),
        py::arg("num_blocks"), py::arg("timing") = py::none(), py::arg("prefetch_ptr") = 0,
        py::arg("prefetch_bytes") = 0);
  m.def("mla_decode", &mla_decode);
  m.def("mla_cache_write", &mla_cache_write);
  m.def("mapped_host_buffer", &mapped_host_buffer);
  m.def("hisparse_resolve", &hisparse_resolve, py::arg("topk"), py::arg("topk_out"), py::arg("q_start"),
        py::arg("seq_lens"), py::arg("state_slots"), py::arg("positions"), py::arg("slot_mapping"),
        py::arg("block_tables"), py::arg("cold"), py::arg("hot"), py::arg("pos2slot"), py::arg("slot2pos"),
        py::arg("stamp"), py::arg("clock"), py::arg("hot_bt"), py::arg("hot_seq"), py::arg("err"),
        py::arg("stats") = py::none());
  m.def("hisparse_reset", &hisparse_reset);
  m.def("dsa_cache_write", &dsa_cache_write);
  m.def("dsa_quant_q", &dsa_quant_q);
  m.def("dsa_index", &dsa_index);
  m.def("gemm_nvfp4", &gemm_nvfp4, py::arg("y"), py::arg("x"), py::arg("packed"), py::arg("scales"),
        py::arg("gscale"), py::arg("bn"), py::arg("groups") = py::none(), py::arg("num_groups") = py::none(),
        py::arg("rows_p") = 0, py::arg("err") = py::none(), py::arg("splits") = 1, py::arg("ws") = py::none());
  m.def("nvfp4_gather_act", &nvfp4_gather_act);
  m.def("nvfp4_quant_act", &nvfp4_quant_act, py::arg("x"), py::arg("xq"), py::arg("x_sf"), py::arg("a_scale"),
        py::arg("tile_rows"), py::arg("static_g") = 0.0, py::arg("groups") = py::none(),
        py::arg("num_groups") = py::none(), py::arg("swiglu") = false);
  m.def("gemm_fp4mma", &gemm_fp4mma, py::arg("y"), py::arg("xq"), py::arg("x_sf"), py::arg("a_scale"), py::arg("w"),
        py::arg("w_sf"), py::arg("alpha_w"), py::arg("bn"), py::arg("groups") = py::none(),
        py::arg("num_groups") = py::none(), py::arg("rows_p") = 0, py::arg("err") = py::none(),
        py::arg("splits") = 1, py::arg("ws") = py::none(), py::arg("counters") = py::none(),
        py::arg("fp8") = false, py::arg("stamps") = py::none());
  m.def("mxfp8_quant_act", &mxfp8_quant_act, py::arg("x"), py::arg("xq"), py::arg("x_sf"), py::arg("a_scale"),
        py::arg("tile_rows"), py::arg("groups") = py::none(), py::arg("num_groups") = py::none());
  m.def("spec_advance", &spec_advance);
  m.def("mla_fp4_row_bytes", [](int64_t cl, int64_t r) { return sh_mla_fp4_row_bytes(cl, r); });
  m.def("gdn_conv", &gdn_conv);
  m.def("gdn_recurrent", &gdn_recurrent);
  m.def("gdn_chunk_prefill", &gdn_chunk_prefill, "Chunked (64-token, tensor-core) GDN prefill from zero state");
  m.def("ep_dispatch", &ep_dispatch, "Expert-parallel dispatch of token rows over NVLink peer memory");
  m.def("ep_combine_push", &ep_combine_push, "Experts' weighted per-token sum stored into the owners' return rows");
  m.def("ep_combine_sum", &ep_combine_sum, "Owner-side sum of the rows pushed by ep_combine_push");
  m.def("ep_combine", &ep_combine, "Expert-parallel combine of expert outputs over NVLink peer memory");
  m.def("moe_route", &moe_route);
  m.def("moe_align", &moe_align);
  m.def("moe_gather", &moe_gather);
  m.def("moe_combine", &moe_combine);
  m.def("gemm_grouped", &gemm_grouped);
  m.def("nvfp4_dequant", &nvfp4_dequant);
  m.def("nvfp4_quant", &nvfp4_quant);
  m.def("gemm_bf16_sk", &gemm_bf16_sk, "stream-K tcgen05 CTA-pair linear", py::arg("y"), py::arg("x"), py::arg("w"),
        py::arg("ns"), py::arg("nsub"), py::arg("clusters"), py::arg("ws"), py::arg("cnt"),
        py::arg("err") = py::none(), py::arg("stamps") = py::none());
  m.def("gemm_sk_max_clusters", &gemm_sk_max_clusters, "co-resident CTA pairs of the stream-K kernel",
        py::arg("ns"), py::arg("nsub"));
  m.def("gemm_bf16", &gemm_bf16, "tcgen05 GEMM", py::arg("y"), py::arg("x"), py::arg("w"), py::arg("swap"),
        py::arg("bn"), py::arg("splits"), py::arg("ws") = py::none(), py::arg("err") = py::none(), py::arg("pair") = false);
}
