"""Checkpoint loading against Hugging Face's own modeling code (CPU, fp32).

A tiny random model of each architecture is built with transformers, saved as
safetensors, loaded into this framework through `config_from_hf` +
`load_weights`, and both greedy-decode the same prompt: the token streams must
be identical.  This checks the name mapping and the layout conversions
(fused QKV / gate-up, Qwen3-Next grouped qkvz / interleaved gate / zero-centred
norms, DeepSeek interleaved rotary rows) as well as RoPE scaling (llama3, YaRN).
Quantised checkpoints (fp8 block-scaled, NVFP4) are checked against their
dequantised values.
"""
import os

import numpy as np
import pytest
import torch

transformers = pytest.importorskip("transformers")


def _hf_greedy(model, prompt, n):
    with torch.no_grad():
        out = model.generate(torch.tensor([prompt]), max_new_tokens=n, do_sample=False, num_beams=1,
                             pad_token_id=0, eos_token_id=None)
    return out[0, len(prompt):].tolist()


def _ours(path, prompt, n):
    from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
    from vllm_suffix_hybrid_b200.engine.loader import config_from_hf
    from vllm_suffix_hybrid_b200.parallel import state

    state._STATE = state.ParallelState()
    m = config_from_hf(path, dtype="float32")
    m.max_position = 512
    eng = LLMEngine(EngineConfig(model=m, spec=SpecConfig(method="none"), cache=CacheConfig(max_model_len=256),
                                 max_num_seqs=2, device="cpu", cuda_graphs=False, weights=path))
    return eng.generate([prompt], n)[0]


def _save(model, tmp_path, name):
    d = str(tmp_path / name)
    model.save_pretrained(d, safe_serialization=True)
    return d


@pytest.mark.parametrize("variant", ["plain", "llama3_rope", "tied"])
def test_llama_matches_hf(tmp_path, variant):
    torch.manual_seed(0)
    kw = dict(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
              num_key_value_heads=2, head_dim=16, rms_norm_eps=1e-5, max_position_embeddings=512, rope_theta=10000.0)
    if variant == "llama3_rope":
        kw["rope_scaling"] = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                              "original_max_position_embeddings": 64}
    if variant == "tied":
        kw["tie_word_embeddings"] = True
    hf = transformers.LlamaForCausalLM(transformers.LlamaConfig(**kw)).float().eval()
    path = _save(hf, tmp_path, variant)
    prompt = list(np.random.default_rng(1).integers(0, 256, 40))
    assert _ours(path, prompt, 16) == _hf_greedy(hf, prompt, 16)


def test_qwen3_next_matches_hf(tmp_path):
    torch.manual_seed(0)
    cfg = transformers.Qwen3NextConfig(vocab_size=256, hidden_size=64, intermediate_size=64, num_hidden_layers=4,
                                       num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                                       linear_num_value_heads=4, linear_num_key_heads=2, linear_key_head_dim=16,
                                       linear_value_head_dim=16, num_experts=4, num_experts_per_tok=2,
                                       moe_intermediate_size=32, shared_expert_intermediate_size=32,
                                       max_position_embeddings=512)
    hf = transformers.Qwen3NextForCausalLM(cfg).float().eval()
    with torch.no_grad():  # zero-centred norm gains are zero at init: make them non-trivial
        for n, p in hf.named_parameters():
            if n.endswith("norm.weight") and "linear_attn.norm" not in n:
                p.normal_(0.0, 0.1)
    path = _save(hf, tmp_path, "qwen3next")
    prompt = list(np.random.default_rng(2).integers(0, 256, 24))
    assert _ours(path, prompt, 10) == _hf_greedy(hf, prompt, 10)


@pytest.mark.parametrize("rope", ["plain", "yarn"])
def test_deepseek_v3_matches_hf(tmp_path, rope):
    torch.manual_seed(0)
    kw = dict(vocab_size=256, hidden_size=64, intermediate_size=96, moe_intermediate_size=32, num_hidden_layers=3,
              num_attention_heads=4, q_lora_rank=32, kv_lora_rank=32, qk_nope_head_dim=16, qk_rope_head_dim=8,
              v_head_dim=16, n_routed_experts=8, num_experts_per_tok=2, n_group=2, topk_group=1, n_shared_experts=1,
              first_k_dense_replace=1, routed_scaling_factor=2.5, norm_topk_prob=True, max_position_embeddings=512,
              rope_theta=10000.0)
    if rope == "yarn":
        kw["rope_scaling"] = {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 128,
                              "beta_fast": 32, "beta_slow": 1, "mscale": 1.0, "mscale_all_dim": 1.0}
    hf = transformers.DeepseekV3ForCausalLM(transformers.DeepseekV3Config(**kw)).float().eval()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if n.endswith("e_score_correction_bias"):
                p.normal_(0.0, 0.05)
    path = _save(hf, tmp_path, "dsv3_" + rope)
    prompt = list(np.random.default_rng(3).integers(0, 256, 24))
    assert _ours(path, prompt, 10) == _hf_greedy(hf, prompt, 10)


def test_yarn_frequencies_match_hf():
    from vllm_suffix_hybrid_b200.ops import reference as ref

    cfg = transformers.DeepseekV3Config(hidden_size=64, num_attention_heads=4, qk_rope_head_dim=8, qk_nope_head_dim=16,
                                        max_position_embeddings=4096,
                                        rope_scaling={"rope_type": "yarn", "factor": 40.0,
                                                      "original_max_position_embeddings": 4096, "beta_fast": 32,
                                                      "beta_slow": 1, "mscale": 1.0, "mscale_all_dim": 1.0})
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    cfg.head_dim = 8
    inv_hf, att_hf = ROPE_INIT_FUNCTIONS["yarn"](cfg, "cpu")
    inv, att = ref.rope_inv_freq(8, 10000.0, cfg.rope_scaling if cfg.rope_scaling else cfg.rope_parameters)
    assert torch.allclose(inv.float(), inv_hf.float(), rtol=1e-5) and abs(att - att_hf) < 1e-6


def test_quantised_checkpoints(tmp_path):
    """fp8 block-scaled and NVFP4 tensors load as their dequantised values."""
    from safetensors.torch import save_file

    from vllm_suffix_hybrid_b200.engine.loader import Checkpoint
    from vllm_suffix_hybrid_b200.ops import reference as ref

    torch.manual_seed(0)
    w = torch.randn(256, 384) * 0.05
    blocks = w.view(2, 128, 3, 128).abs().amax(dim=(1, 3)) / 448.0
    q = (w / blocks.repeat_interleave(128, 0).repeat_interleave(128, 1)).to(torch.float8_e4m3fn)
    g = ref.nvfp4_global_scale(w)
    packed, scales = ref.nvfp4_quantize(w.to(torch.bfloat16), g)
    save_file({"a.weight": q, "a.weight_scale_inv": blocks, "b.weight": packed, "b.weight_scale": scales,
               "b.weight_scale_2": g}, str(tmp_path / "m.safetensors"))
    ck = Checkpoint(str(tmp_path))
    a = ck.matrix("a")
    assert torch.allclose(a, q.float() * blocks.repeat_interleave(128, 0).repeat_interleave(128, 1))
    assert bool(((a - w).abs() <= 0.07 * w.abs() + 1e-3).all())  # e4m3: 3 mantissa bits
    b = ck.matrix("b")
    assert torch.equal(b, ref.nvfp4_dequantize(packed, scales, g).float())
    assert ck.is_nvfp4("b") and not ck.is_nvfp4("a")


def test_nvfp4_writer_roundtrip(tmp_path):
    """quantize.convert writes a ModelOpt NVFP4 checkpoint that the loader reads back: the codes and
    scales equal the reference quantiser's, fused groups share weight_scale_2, and the loaded model
    generates from the dequantised weights."""
    import json as _json

    from vllm_suffix_hybrid_b200.engine import quantize
    from vllm_suffix_hybrid_b200.engine.loader import Checkpoint
    from vllm_suffix_hybrid_b200.ops import reference as ref

    torch.manual_seed(0)
    cfg = transformers.LlamaConfig(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, head_dim=16)
    hf = transformers.LlamaForCausalLM(cfg).float().eval()
    src = _save(hf, tmp_path, "bf16")
    out = str(tmp_path / "nvfp4")
    stats = quantize.convert(src, out)
    assert stats["quantized"] == 2 * 7
    ck = Checkpoint(out)
    base = "model.layers.0.self_attn.q_proj"
    assert ck.is_nvfp4(base)
    g_q = float(ck.get(base + ".weight_scale_2"))
    g_k = float(ck.get("model.layers.0.self_attn.k_proj.weight_scale_2"))
    assert g_q == g_k  # q|k|v share one global scale
    w = hf.model.layers[0].self_attn.q_proj.weight.detach()
    p_ref, s_ref = ref.nvfp4_quantize(w, torch.tensor([g_q]))
    assert torch.equal(ck.get(base + ".weight"), p_ref)
    assert torch.equal(ck.get(base + ".weight_scale").view(torch.uint8), s_ref.view(torch.uint8))
    assert _json.load(open(os.path.join(out, "hf_quant_config.json")))["quantization"]["quant_algo"] == "NVFP4"
    # the quantised model loads and runs (dequantised weights in bf16/fp32 layers)
    prompt = list(range(10, 30))
    toks = _ours(out, prompt, 6)
    assert len(toks) == 6
