"""Hugging Face safetensors checkpoints: config and weights (bf16/fp16/fp32, fp8 block-scaled, NVFP4).

Formats, detected per tensor:
* plain floating point -> cast to the model dtype;
* fp8 e4m3 with ``<name>_scale_inv`` [ceil(N/b), ceil(K/b)] (DeepSeek block scaling, b = 128)
  or a per-tensor ``<name>_scale`` -> dequantised;
* NVFP4 in the ModelOpt layout (reference: suffix_hybrid/tools/quantize_nvfp4.py):
  ``weight`` uint8 [N, K/2] (two e2m1 codes, low nibble first), ``weight_scale`` e4m3 [N, K/16],
  ``weight_scale_2`` fp32 -> kept packed by NVFP4 layers, dequantised for bf16 layers.

Architectures (name layout of the HF modeling code): LlamaForCausalLM (+ an EAGLE /
MTP draft head under ``draft.`` / ``mtp.`` when present), Qwen3NextForCausalLM (+ ``mtp.``),
DeepseekV3ForCausalLM / Kimi-K2 / DeepSeek-V3.2 (+ the MTP layer ``model.layers.<L>``).
Layout conversions done here, once, at load:
* fused q|k|v and gate|up matrices are concatenated, then sliced per TP rank;
* Qwen3-Next ``in_proj_qkvz`` / ``in_proj_ba`` rows are grouped per key head in the checkpoint
  and regrouped to [q | k | v | z] / [b | a]; ``q_proj`` interleaves query and gate per head;
  its zero-centred RMSNorm gains are stored as (gain - 1);
* DeepSeek rotary channels are stored as interleaved pairs: the rope rows of ``q_b_proj`` and
  ``kv_a_proj_with_mqa`` are de-interleaved so the rotate-half RoPE gives the same dot products.
"""
from __future__ import annotations

import json
import logging
import os
from typing import Dict, Optional

import torch

logger = logging.getLogger("suffix_hybrid.loader")


# ------------------------------------------------------------------------------------------ files
class Checkpoint:
    def __init__(self, path: str):
        from safetensors import safe_open

        self.path = path
        files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
        if not files:
            raise FileNotFoundError(f"no .safetensors files in {path}")
        self._open = {}
        self._where: Dict[str, str] = {}
        for f in files:
            h = safe_open(os.path.join(path, f), framework="pt")
            self._open[f] = h
            for k in h.keys():
                self._where[k] = f
        self.used = set()

    def has(self, name: str) -> bool:
        return name in self._where

    def get(self, name: str) -> torch.Tensor:
        if name not in self._where:
            raise KeyError(f"{name} not in checkpoint {self.path}")
        self.used.add(name)
        return self._open[self._where[name]].get_tensor(name)

    def names(self):
        return self._where.keys()

    def is_nvfp4(self, base: str) -> bool:
        return self.has(base + ".weight_scale_2") and self.has(base + ".weight_scale")

    def matrix(self, base: str) -> torch.Tensor:
        """Full [out, in] float32 matrix of `<base>.weight` in any supported format."""
        from ..ops import reference as ref

        w = self.get(base + ".weight")
        if self.is_nvfp4(base) and w.dtype == torch.uint8:
            return ref.nvfp4_dequantize(w, self.get(base + ".weight_scale"), self.get(base + ".weight_scale_2")).float()
        if w.dtype == torch.float8_e4m3fn:
            if self.has(base + ".weight_scale_inv"):
                s = self.get(base + ".weight_scale_inv").float()
                N, K = w.shape
                bn, bk = -(-N // s.shape[0]), -(-K // s.shape[1])
                full = s.repeat_interleave(bn, 0)[:N].repeat_interleave(bk, 1)[:, :K]
                return w.float() * full
            if self.has(base + ".weight_scale"):
                return w.float() * self.get(base + ".weight_scale").float().reshape(-1)[0]
            return w.float()
        return w.float()

    def nvfp4(self, base: str):
        return (self.get(base + ".weight"), self.get(base + ".weight_scale"),
                self.get(base + ".weight_scale_2").float().reshape(1))

    def unused(self):
        return sorted(set(self._where) - self.used)


# ------------------------------------------------------------------------------------------ config
def _rope(hf: dict):
    rp = hf.get("rope_parameters") or {}
    theta = float(rp.get("rope_theta", hf.get("rope_theta", 10000.0)))
    scaling = hf.get("rope_scaling") or (rp if rp.get("rope_type", "default") != "default" else None)
    if scaling is not None and scaling.get("rope_type", scaling.get("type", "default")) == "default":
        scaling = None
    prf = float(rp.get("partial_rotary_factor", hf.get("partial_rotary_factor", 1.0)))
    return theta, (dict(scaling) if scaling else None), prf


def config_from_hf(path_or_dict, dtype: str = "bfloat16"):
    """ModelConfig of a Hugging Face checkpoint directory (config.json) or config dict."""
    from .config import ModelConfig

    hf = path_or_dict
    if isinstance(path_or_dict, str):
        with open(os.path.join(path_or_dict, "config.json")) as f:
            hf = json.load(f)
    arch = (hf.get("architectures") or [""])[0]
    mt = hf.get("model_type", "")
    theta, scaling, prf = _rope(hf)
    common = dict(hidden=hf["hidden_size"], layers=hf["num_hidden_layers"], heads=hf["num_attention_heads"],
                  vocab=hf["vocab_size"], rope_theta=theta, rope_scaling=scaling,
                  norm_eps=float(hf.get("rms_norm_eps", 1e-6)),
                  max_position=int(hf.get("max_position_embeddings", 8192)),
                  tie_embeddings=bool(hf.get("tie_word_embeddings", False)), dtype=dtype)
    quant = (hf.get("quantization_config") or {})
    fmt = "bf16"
    if quant.get("quant_method") == "fp8":
        fmt = "fp8_block"
    elif "nvfp4" in json.dumps(quant).lower() or os.path.exists(os.path.join(str(path_or_dict), "hf_quant_config.json")):
        fmt = "nvfp4"
    if mt == "llama" or arch == "LlamaForCausalLM":
        return ModelConfig(arch="llama", kv_heads=hf.get("num_key_value_heads", hf["num_attention_heads"]),
                           head_dim=hf.get("head_dim") or hf["hidden_size"] // hf["num_attention_heads"],
                           ffn=hf["intermediate_size"], weight_format=fmt, draft="eagle", **common)
    if mt == "qwen3_next" or arch == "Qwen3NextForCausalLM":
        lt = hf.get("layer_types")
        interval = int(hf.get("full_attention_interval", 4))
        pattern = "".join("A" if t == "full_attention" else "L" for t in lt) if lt else "L" * (interval - 1) + "A"
        return ModelConfig(arch="qwen3_next", kv_heads=hf["num_key_value_heads"], head_dim=hf["head_dim"],
                           ffn=hf.get("intermediate_size", 0), num_experts=hf["num_experts"],
                           top_k=hf["num_experts_per_tok"], expert_ffn=hf["moe_intermediate_size"],
                           shared_experts=1 if hf.get("shared_expert_intermediate_size") else 0,
                           shared_ffn=hf.get("shared_expert_intermediate_size", 0), router="softmax",
                           layer_pattern=pattern, gdn_qk_heads=hf["linear_num_key_heads"],
                           gdn_v_heads=hf["linear_num_value_heads"], gdn_head_dim=hf["linear_key_head_dim"],
                           gdn_conv=hf.get("linear_conv_kernel_dim", 4), attn_gated=True, partial_rotary=prf,
                           norm_offset=1.0, weight_format=fmt, draft="mtp", **common)
    if mt in ("deepseek_v3", "deepseek_v32", "kimi_k2") or arch in ("DeepseekV3ForCausalLM", "DeepseekV32ForCausalLM"):
        v32 = mt == "deepseek_v32" or "index_topk" in hf
        return ModelConfig(arch="deepseek_v32" if v32 else "kimi_k2", kv_heads=1,
                           head_dim=hf["qk_nope_head_dim"] + hf["qk_rope_head_dim"], ffn=hf["intermediate_size"],
                           num_experts=hf.get("n_routed_experts") or 0, top_k=hf.get("num_experts_per_tok") or 0,
                           expert_ffn=hf.get("moe_intermediate_size") or 0,
                           shared_experts=hf.get("n_shared_experts") or 0,
                           shared_ffn=(hf.get("moe_intermediate_size") or 0) * (hf.get("n_shared_experts") or 0),
                           router="sigmoid_grouped", n_groups=hf.get("n_group") or 1,
                           topk_groups=hf.get("topk_group") or 1,
                           routed_scale=float(hf.get("routed_scaling_factor", 1.0)),
                           first_dense_layers=hf.get("first_k_dense_replace", 0), q_lora=hf.get("q_lora_rank") or 0,
                           kv_lora=hf["kv_lora_rank"], qk_nope=hf["qk_nope_head_dim"], qk_rope=hf["qk_rope_head_dim"],
                           v_head=hf["v_head_dim"], dsa_heads=hf.get("index_n_heads", 0) if v32 else 0,
                           dsa_head_dim=hf.get("index_head_dim", 128), dsa_topk=hf.get("index_topk", 0) if v32 else 0,
                           weight_format=fmt, draft="mtp", **common)
    raise ValueError(f"unsupported checkpoint architecture {arch or mt!r}")


# ------------------------------------------------------------------------------------------ helpers
def _copy(dst: torch.Tensor, src: torch.Tensor, what: str) -> None:
    if tuple(dst.shape) != tuple(src.shape):
        raise ValueError(f"{what}: checkpoint shape {tuple(src.shape)} != model {tuple(dst.shape)}")
    dst.copy_(src.to(device=dst.device, dtype=dst.dtype))


def _norm(ck: Checkpoint, name: str, norm, offset: float = 0.0) -> None:
    _copy(norm.weight, ck.get(name).float() + offset, name)


def _deinterleave_rows(w: torch.Tensor, start: int, n: int, period: Optional[int] = None) -> torch.Tensor:
    """Reorder rows [start, start+n) (every `period` rows when given) from interleaved pairs to halves."""
    w = w.clone()
    perm = torch.cat([torch.arange(0, n, 2), torch.arange(1, n, 2)])
    starts = [start] if period is None else list(range(start, w.shape[0], period))
    for s0 in starts:
        w[s0:s0 + n] = w[s0:s0 + n][perm]
    return w


def _moe(ck: Checkpoint, pre: str, moe, shared_name: str) -> None:
    from ..parallel import state

    st = state.get()
    _copy(moe.gate, ck.get(pre + "gate.weight").float(), pre + "gate")
    if moe.bias is not None and ck.has(pre + "gate.e_score_correction_bias"):
        _copy(moe.bias, ck.get(pre + "gate.e_score_correction_bias").float(), pre + "bias")
    F, H = moe.F, moe.H
    e0 = st.ep_rank * moe.E_local if moe.ep > 1 else 0
    for j in range(moe.E_local):
        e = e0 + j
        base = f"{pre}experts.{e}."
        if getattr(moe, "fp4", None) is not None:
            _fp4_expert(ck, moe, j, base)
            continue
        if getattr(moe, "fp8", None) is not None:
            _fp8_expert(ck, moe, j, base)
            continue
        g = ck.matrix(base + "gate_proj")
        u = ck.matrix(base + "up_proj")
        d = ck.matrix(base + "down_proj")
        _copy(moe.w13[j * 2 * F:(j + 1) * 2 * F], torch.cat([g, u], 0), f"{pre}experts.{e}.gate|up")
        _copy(moe.w2[j * H:(j + 1) * H], d, f"{pre}experts.{e}.down")
    if getattr(moe, "fp4", None) is not None:
        moe.refresh()
    if getattr(moe, "fp8", None) is not None:  # scale tiles of the re-quantised experts
        from .. import ops

        moe.fp8 = tuple((c, sc, ops.mxfp8_scale_tiles(sc, r)) for (c, sc, _), r in zip(moe.fp8, (2 * moe.F, moe.H)))
    if moe.shared is not None:
        sp = pre + shared_name + "."
        moe.shared.gate_up.load(torch.cat([ck.matrix(sp + "gate_proj"), ck.matrix(sp + "up_proj")], 0))
        moe.shared.down.load(ck.matrix(sp + "down_proj"))
    if moe.shared_gate is not None:
        _copy(moe.shared_gate, ck.get(pre + "shared_expert_gate.weight").float(), pre + "shared_expert_gate")


def _fp8_expert(ck: Checkpoint, moe, j: int, base: str) -> None:
    """Fill MXFP8 expert j from the checkpoint's (dequantised) matrices: per-32 e4m3 + ue8m0.  Power-of-two
    block scales (ue8m0 checkpoints) re-quantise exactly; other block scales round once more."""
    from .. import ops

    F, H = moe.F, moe.H
    (c13, s13, _), (c2, s2, _) = moe.fp8
    w = torch.cat([ck.matrix(base + "gate_proj"), ck.matrix(base + "up_proj")]).to(c13.device)
    c, sc = ops.mxfp8_quantize(w)
    c13[j * 2 * F:(j + 1) * 2 * F], s13[j * 2 * F:(j + 1) * 2 * F] = c, sc
    c, sc = ops.mxfp8_quantize(ck.matrix(base + "down_proj").to(c2.device))
    c2[j * H:(j + 1) * H], s2[j * H:(j + 1) * H] = c, sc


def _fp4_expert(ck: Checkpoint, moe, j: int, base: str) -> None:
    """Fill NVFP4 expert j: copy ModelOpt-packed tensors when gate and up share one global scale,
    otherwise quantise the (dequantised) full matrices."""
    from .. import ops

    F, H = moe.F, moe.H
    (p13, s13, g13), (p2, s2, g2) = moe.fp4[0][:3], moe.fp4[1][:3]
    gname, uname, dname = base + "gate_proj", base + "up_proj", base + "down_proj"
    if ck.is_nvfp4(gname) and ck.is_nvfp4(uname) and \
            float(ck.get(gname + ".weight_scale_2")) == float(ck.get(uname + ".weight_scale_2")):
        pg, sg, gg = ck.nvfp4(gname)
        pu, su, _ = ck.nvfp4(uname)
        p13[j * 2 * F:(j + 1) * 2 * F] = torch.cat([pg, pu]).to(p13.device)
        s13[j * 2 * F:(j + 1) * 2 * F] = torch.cat([sg, su]).to(s13.device)
        g13[j] = gg.to(g13.device)[0]
    else:
        w = torch.cat([ck.matrix(gname), ck.matrix(uname)]).to(p13.device, torch.bfloat16)
        p, sc, g = ops.nvfp4_quantize(w)
        p13[j * 2 * F:(j + 1) * 2 * F], s13[j * 2 * F:(j + 1) * 2 * F], g13[j] = p, sc, g.reshape(-1)[0]
    if ck.is_nvfp4(dname):
        pd, sd, gd = ck.nvfp4(dname)
        p2[j * H:(j + 1) * H], s2[j * H:(j + 1) * H], g2[j] = pd.to(p2.device), sd.to(s2.device), gd.to(g2.device)[0]
    else:
        p, sc, g = ops.nvfp4_quantize(ck.matrix(dname).to(p2.device, torch.bfloat16))
        p2[j * H:(j + 1) * H], s2[j * H:(j + 1) * H], g2[j] = p, sc, g.reshape(-1)[0]


def _mlp(ck: Checkpoint, pre: str, mlp) -> None:
    mlp.gate_up.load(torch.cat([ck.matrix(pre + "gate_proj"), ck.matrix(pre + "up_proj")], 0))
    mlp.down.load(ck.matrix(pre + "down_proj"))


# ------------------------------------------------------------------------------------------ llama
def _llama_layer(ck: Checkpoint, pre: str, layer, with_input_norm: bool = True) -> None:
    if with_input_norm:
        _norm(ck, pre + "input_layernorm.weight", layer.input_norm)
    a = pre + "self_attn."
    layer.attn.qkv.load(torch.cat([ck.matrix(a + "q_proj"), ck.matrix(a + "k_proj"), ck.matrix(a + "v_proj")], 0))
    layer.attn.o.load(ck.matrix(a + "o_proj"))
    _norm(ck, pre + "post_attention_layernorm.weight", layer.post_norm)
    _mlp(ck, pre + "mlp.", layer.mlp)


def _load_llama(ck: Checkpoint, model, draft) -> None:
    _copy(model.embed, ck.get("model.embed_tokens.weight").float(), "embed")
    for i, layer in enumerate(model.layers):
        _llama_layer(ck, f"model.layers.{i}.", layer)
    _norm(ck, "model.norm.weight", model.norm)
    model.lm_head.load(ck.matrix("lm_head") if ck.has("lm_head.weight") else ck.get("model.embed_tokens.weight").float())
    if draft is not None:
        for pre in ("draft.", "mtp.", "eagle."):
            if ck.has(pre + "fc.weight"):
                _copy(draft.fc, ck.matrix(pre + "fc"), pre + "fc")
                lp = pre + "layers.0."
                _llama_layer(ck, lp, draft.layer, with_input_norm=ck.has(lp + "input_layernorm.weight"))
                for nm, norm in (("enorm", draft.enorm), ("hnorm", draft.hnorm), ("norm", draft.norm)):
                    if ck.has(pre + nm + ".weight"):
                        _norm(ck, pre + nm + ".weight", norm)
                break
        else:
            logger.warning("checkpoint has no draft head weights (draft./mtp./eagle. prefixes): keeping random init")


# ------------------------------------------------------------------------------------------ qwen3-next
def _qwen_attn(ck: Checkpoint, pre: str, attn, cfg) -> None:
    a = pre + "self_attn."
    H, D = cfg.heads, cfg.head_dim
    qg = ck.matrix(a + "q_proj").view(H, 2, D, -1)  # per head: [query D | gate D]
    q, gate = qg[:, 0].reshape(H * D, -1), qg[:, 1].reshape(H * D, -1)
    attn.qkvg.load(torch.cat([q, ck.matrix(a + "k_proj"), ck.matrix(a + "v_proj"), gate], 0))
    attn.o.load(ck.matrix(a + "o_proj"))
    _norm(ck, a + "q_norm.weight", attn.q_norm, cfg.norm_offset)
    _norm(ck, a + "k_norm.weight", attn.k_norm, cfg.norm_offset)


def _qwen_gdn(ck: Checkpoint, pre: str, gdn, cfg) -> None:
    a = pre + "linear_attn."
    H, HV, K = gdn.H, gdn.HV, gdn.K
    rep = HV // H
    w = ck.matrix(a + "in_proj_qkvz").view(H, 2 * K + 2 * rep * K, -1)
    q, k = w[:, :K], w[:, K:2 * K]
    v, z = w[:, 2 * K:2 * K + rep * K], w[:, 2 * K + rep * K:]
    flat = lambda t: t.reshape(-1, t.shape[-1])
    gdn.in_qkvz.load(torch.cat([flat(q), flat(k), flat(v), flat(z)], 0))
    ba = ck.matrix(a + "in_proj_ba").view(H, 2 * rep, -1)
    gdn.in_ba.load(torch.cat([flat(ba[:, :rep]), flat(ba[:, rep:])], 0))
    _copy(gdn.conv_w, ck.get(a + "conv1d.weight").float().reshape(gdn.C, -1), a + "conv1d")
    _copy(gdn.a_log, ck.get(a + "A_log").float(), a + "A_log")
    _copy(gdn.dt_bias, ck.get(a + "dt_bias").float(), a + "dt_bias")
    _copy(gdn.norm_w, ck.get(a + "norm.weight").float(), a + "norm")
    gdn.out.load(ck.matrix(a + "out_proj"))


def _qwen_layer(ck: Checkpoint, pre: str, layer, cfg) -> None:
    _norm(ck, pre + "input_layernorm.weight", layer.input_norm, cfg.norm_offset)
    if layer.kind == "L":
        _qwen_gdn(ck, pre, layer.mixer, cfg)
    else:
        _qwen_attn(ck, pre, layer.mixer, cfg)
    _norm(ck, pre + "post_attention_layernorm.weight", layer.post_norm, cfg.norm_offset)
    _moe(ck, pre + "mlp.", layer.moe, "shared_expert")


def _load_qwen3_next(ck: Checkpoint, model, draft) -> None:
    cfg = model.cfg
    _copy(model.embed, ck.get("model.embed_tokens.weight").float(), "embed")
    for i, layer in enumerate(model.layers):
        _qwen_layer(ck, f"model.layers.{i}.", layer, cfg)
    _norm(ck, "model.norm.weight", model.norm, cfg.norm_offset)
    model.lm_head.load(ck.matrix("lm_head") if ck.has("lm_head.weight") else ck.get("model.embed_tokens.weight").float())
    if draft is not None:
        if ck.has("mtp.fc.weight"):
            _copy(draft.fc, ck.matrix("mtp.fc"), "mtp.fc")
            _norm(ck, "mtp.pre_fc_norm_embedding.weight", draft.enorm, cfg.norm_offset)
            _norm(ck, "mtp.pre_fc_norm_hidden.weight", draft.hnorm, cfg.norm_offset)
            _qwen_layer(ck, "mtp.layers.0.", draft.layer, cfg)
            _norm(ck, "mtp.norm.weight", draft.norm, cfg.norm_offset)
        else:
            logger.warning("checkpoint has no mtp.* weights: keeping the MTP head's random init")


# ------------------------------------------------------------------------------------------ deepseek
def _qlinear(ck: Checkpoint, base: str, lin, transform=None) -> None:
    if lin.fmt == "nvfp4" and ck.is_nvfp4(base) and transform is None:
        p, s, g = ck.nvfp4(base)
        lin.packed.copy_(p.to(lin.packed.device))
        lin.scales.copy_(s.to(lin.scales.device))
        lin.gscale.copy_(g.to(lin.gscale.device))
        if ck.has(base + ".input_scale"):  # static activation scale of the W4A4 path
            isc = float(ck.get(base + ".input_scale").float().reshape(-1).max())
            lin.static_g = 1.0 / isc if isc > 0 else 0.0
        lin.refresh()
        return
    full = ck.matrix(base)
    if transform is not None:
        full = transform(full)
    lin.load(full)


def _ds_layer(ck: Checkpoint, pre: str, layer, cfg) -> None:
    a = pre + "self_attn."
    att = layer.attn
    _norm(ck, pre + "input_layernorm.weight", layer.input_norm)
    nope, rope = cfg.qk_nope, cfg.qk_rope
    if att.q_a is not None:
        _qlinear(ck, a + "q_a_proj", att.q_a)
        _norm(ck, a + "q_a_layernorm.weight", att.q_a_norm)
        _qlinear(ck, a + "q_b_proj", att.q_b, lambda w: _deinterleave_rows(w, nope, rope, nope + rope))
    else:
        _qlinear(ck, a + "q_proj", att.q_b, lambda w: _deinterleave_rows(w, nope, rope, nope + rope))
    _qlinear(ck, a + "kv_a_proj_with_mqa", att.kv_a, lambda w: _deinterleave_rows(w, cfg.kv_lora, rope))
    _norm(ck, a + "kv_a_layernorm.weight", att.kv_a_norm)
    _qlinear(ck, a + "kv_b_proj", att.kv_b)
    _qlinear(ck, a + "o_proj", att.o)
    if att.dsa:
        ip = a + "indexer."
        _qlinear(ck, ip + "wq_b", att.idx_q)
        _qlinear(ck, ip + "wk", att.idx_k)
        _copy(att.idx_w, ck.matrix(ip + "weights_proj"), ip + "weights_proj")
    _norm(ck, pre + "post_attention_layernorm.weight", layer.post_norm)
    if hasattr(layer.ffn, "w13"):
        _moe(ck, pre + "mlp.", layer.ffn, "shared_experts")
    else:
        _mlp(ck, pre + "mlp.", layer.ffn)


def _load_deepseek(ck: Checkpoint, model, draft) -> None:
    cfg = model.cfg
    _copy(model.embed, ck.get("model.embed_tokens.weight").float(), "embed")
    for i, layer in enumerate(model.layers):
        _ds_layer(ck, f"model.layers.{i}.", layer, cfg)
    _norm(ck, "model.norm.weight", model.norm)
    model.lm_head.load(ck.matrix("lm_head"))
    if draft is not None:
        pre = f"model.layers.{cfg.layers}."
        if ck.has(pre + "eh_proj.weight"):
            _copy(draft.eh_proj, ck.matrix(pre + "eh_proj"), pre + "eh_proj")
            _norm(ck, pre + "enorm.weight", draft.enorm)
            _norm(ck, pre + "hnorm.weight", draft.hnorm)
            _ds_layer(ck, pre, draft.layer, cfg)
            _norm(ck, pre + "shared_head.norm.weight", draft.norm)
        else:
            logger.warning("checkpoint has no MTP layer (%seh_proj): keeping random init", pre)


# ------------------------------------------------------------------------------------------ entry
def load_weights(model, draft, path: str, strict: bool = False) -> Checkpoint:
    """Load a checkpoint directory into `model` (and its draft head). Returns the opened checkpoint."""
    ck = Checkpoint(path)
    arch = model.cfg.arch
    with torch.no_grad():
        if arch == "llama":
            _load_llama(ck, model, draft)
        elif arch == "qwen3_next":
            _load_qwen3_next(ck, model, draft)
        elif arch in ("deepseek_v32", "kimi_k2"):
            _load_deepseek(ck, model, draft)
        else:
            raise ValueError(f"no loader for architecture {arch!r}")
    left = [n for n in ck.unused() if not n.endswith(("rotary_emb.inv_freq", "input_scale"))]
    if left:
        msg = f"{len(left)} checkpoint tensors were not used, e.g. {left[:5]}"
        if strict:
            raise ValueError(msg)
        logger.warning(msg)
    return ck
