"""Write an NVFP4 (ModelOpt layout) checkpoint from a bf16/fp16/fp32 safetensors checkpoint.

  python -m vllm_suffix_hybrid_b200.engine.quantize --src DIR --out DIR [--scale-search mse] [--device cuda]

Behaviour of the reference's writer (reference: suffix_hybrid/tools/quantize_nvfp4.py):
* only allow-listed decoder linears are quantised (attention q/k/v/o, dense MLP gate/up/down,
  linear-attention in_proj_qkv(z)/in_proj_z/out_proj); with --experts (default on) also the
  routed / shared MoE experts and the MLA projections; everything else (embeddings, lm_head,
  norms, gates, conv, MTP) is copied unchanged;
* per tensor: uint8 [N, K/2] (two e2m1 codes, element 2i in the low nibble), e4m3 block-16
  scales [N, K/16], fp32 ``weight_scale_2`` = group amax / (6 * 448); tensors that a consumer
  fuses (q|k|v, gate|up, in_proj_qkv|in_proj_z) share one ``weight_scale_2``;
* block scale = e4m3(block max / c / weight_scale_2), c = 6, or with ``--scale-search mse`` the
  c in {6, 5, 4.5, 4} with the lowest squared error per block; codes are the nearest e2m1
  magnitude, exact midpoints to the even code;
* ``input_scale`` (activation scale for W4A4 consumers) is written from ``--act-amax`` (a
  single calibrated activation |x| max, default 448 * 6 = 2688, i.e. scale 1.0): this framework's
  kernels run the NVFP4 weights against bf16 activations and do not read it;
* config.json gains ``quantization_config``; hf_quant_config.json (quant_algo NVFP4, group 16,
  exclude_modules) and a manifest with the source files' sha256 are written; other side files
  (tokenizer, templates) are copied.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import re
import shutil
from typing import Dict, Tuple

import torch

GROUP = 16
FP4_MAX, E4M3_MAX = 6.0, 448.0
GLOBAL = FP4_MAX * E4M3_MAX
EXCLUDE = ["lm_head", "embed_tokens", "mtp", "in_proj_b", "in_proj_a", "in_proj_ba", "gate.weight",
           "shared_expert_gate", "visual", "vision", "audio", "per_layer"]
_BASE = r"^(?:model\.language_model\.|language_model\.model\.|model\.)?layers\.(\d+)\."
DENSE_RE = re.compile(_BASE + r"(self_attn\.(?:q_proj|k_proj|v_proj|o_proj)|mlp\.(?:gate_proj|up_proj|down_proj)"
                      r"|linear_attn\.(?:in_proj_qkvz|in_proj_qkv|in_proj_z|out_proj))\.weight$")
EXPERT_RE = re.compile(_BASE + r"(mlp\.(?:experts\.\d+|shared_experts?)\.(?:gate_proj|up_proj|down_proj)"
                       r"|self_attn\.(?:q_a_proj|q_b_proj|kv_a_proj_with_mqa|kv_b_proj))\.weight$")
FUSED = {"q_proj": "qkv", "k_proj": "qkv", "v_proj": "qkv", "gate_proj": "gate_up", "up_proj": "gate_up",
         "in_proj_qkv": "in_proj_qkvz", "in_proj_z": "in_proj_qkvz"}
COPY_EXT = (".json", ".jinja", ".txt", ".model", ".tiktoken", ".py")


def classify(key: str, experts: bool):
    """Fused-group name of an allow-listed weight, else None."""
    m = DENSE_RE.match(key) or (EXPERT_RE.match(key) if experts else None)
    if not m or any(x in key for x in ("mtp.",)):
        return None
    base = key[: -len(".weight")]
    head, _, leaf = base.rpartition(".")
    return head + "." + FUSED.get(leaf, leaf)


def e2m1_codes(x: torch.Tensor) -> torch.Tensor:
    a = x.abs().clamp(max=FP4_MAX)
    mids = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], device=x.device)
    odd = torch.tensor([False, True, False, True, False, True, False], device=x.device)
    code = ((a[..., None] > mids).sum(-1) + ((a[..., None] == mids) & odd).sum(-1)).to(torch.uint8)
    return code | ((x < 0).to(torch.uint8) << 3)


def quantize(w: torch.Tensor, amax: float, search=(FP4_MAX,)):
    """(packed uint8 [N, K/2], scales e4m3 [N, K/16], weight_scale_2 fp32 []) of w [N, K]."""
    n, k = w.shape
    if k % GROUP:
        raise ValueError(f"K={k} is not a multiple of {GROUP}")
    # fp32 arithmetic in the same order as the loader-side reference quantiser
    ws2 = torch.tensor(max(float(amax), 1e-12) / GLOBAL, dtype=torch.float32, device=w.device)
    blk = w.float().reshape(n, k // GROUP, GROUP)
    bmax = blk.abs().amax(-1)
    lut = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6], dtype=torch.float32, device=w.device)
    best = None
    for c in search:
        sf = (bmax / c / ws2).clamp(max=E4M3_MAX).to(torch.float8_e4m3fn)
        sff = sf.float() * ws2
        code = e2m1_codes(blk / torch.where(sff > 0, sff, torch.ones_like(sff))[..., None])
        if len(search) == 1:
            best = (None, sf, code)
            break
        val = lut[(code & 7).long()] * torch.where(code & 8 > 0, -1.0, 1.0)
        err = ((val * sff[..., None] - blk) ** 2).sum(-1)
        if best is None:
            best = (err, sf, code)
        else:
            take = err < best[0]
            best = (torch.where(take, err, best[0]), torch.where(take, sf, best[1]),
                    torch.where(take[..., None], code, best[2]))
    code = best[2].reshape(n, k)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).contiguous()
    return packed, best[1].contiguous(), ws2.cpu()


def _sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def convert(src: str, out: str, search=(FP4_MAX,), experts: bool = True, device: str = "cpu",
            act_amax: float = GLOBAL, shard_bytes: int = 4 << 30) -> Dict[str, int]:
    from safetensors import safe_open
    from safetensors.torch import save_file

    os.makedirs(out, exist_ok=True)
    files = sorted(f for f in os.listdir(src) if f.endswith(".safetensors"))
    amax: Dict[str, float] = {}
    for f in files:  # pass 1: fused-group |w| max
        with safe_open(os.path.join(src, f), "pt") as st:
            for key in st.keys():
                g = classify(key, experts)
                if g is not None:
                    amax[g] = max(amax.get(g, 0.0), float(st.get_tensor(key).float().abs().amax()))
    weight_map: Dict[str, str] = {}
    stats = {"quantized": 0, "copied": 0}
    shard: Dict[str, torch.Tensor] = {}
    size, idx = 0, 0

    def flush():
        nonlocal shard, size, idx
        if not shard:
            return
        idx += 1
        name = f"model-{idx:05d}.safetensors"
        save_file(shard, os.path.join(out, name), metadata={"format": "pt"})
        for k in shard:
            weight_map[k] = name
        shard, size = {}, 0

    for f in files:  # pass 2: quantise / copy
        with safe_open(os.path.join(src, f), "pt") as st:
            for key in st.keys():
                t = st.get_tensor(key)
                g = classify(key, experts)
                if g is None or t.dim() != 2 or t.shape[1] % GROUP:
                    shard[key] = t
                    stats["copied"] += 1
                    size += t.numel() * t.element_size()
                else:
                    base = key[: -len(".weight")]
                    p, sf, ws2 = quantize(t.to(device), amax[g], search)
                    shard[base + ".weight"] = p.cpu()
                    shard[base + ".weight_scale"] = sf.cpu()
                    shard[base + ".weight_scale_2"] = ws2
                    shard[base + ".input_scale"] = torch.tensor(act_amax / GLOBAL, dtype=torch.float32)
                    stats["quantized"] += 1
                    size += p.numel() + sf.numel() + 8
                if size >= shard_bytes:
                    flush()
    flush()
    with open(os.path.join(out, "model.safetensors.index.json"), "w") as fh:
        json.dump({"metadata": {}, "weight_map": weight_map}, fh, indent=1)
    qcfg = {"quant_method": "modelopt", "producer": {"name": "vllm_suffix_hybrid_b200.engine.quantize"},
            "quantization": {"quant_algo": "NVFP4", "group_size": GROUP, "kv_cache_quant_algo": None,
                             "exclude_modules": EXCLUDE}}
    for name in os.listdir(src):
        if name.endswith(COPY_EXT) and not name.endswith(".safetensors.index.json"):
            shutil.copy(os.path.join(src, name), os.path.join(out, name))
    cfg_path = os.path.join(out, "config.json")
    if os.path.exists(cfg_path):
        with open(cfg_path) as fh:
            cfg = json.load(fh)
        cfg["quantization_config"] = {"quant_method": "modelopt", "quant_algo": "NVFP4", "group_size": GROUP,
                                      "exclude_modules": EXCLUDE}
        with open(cfg_path, "w") as fh:
            json.dump(cfg, fh, indent=2)
    with open(os.path.join(out, "hf_quant_config.json"), "w") as fh:
        json.dump(qcfg, fh, indent=1)
    manifest = {"sources": {f: _sha256(os.path.join(src, f)) for f in files}, "stats": stats,
                "recipe": {"scale_search": list(search), "experts": experts, "act_amax": act_amax}}
    with open(os.path.join(out, "suffix_quant_manifest.json"), "w") as fh:
        json.dump(manifest, fh, indent=1)
    return stats


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="vllm_suffix_hybrid_b200.engine.quantize")
    ap.add_argument("--src", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--scale-search", default="none", choices=["none", "mse"])
    ap.add_argument("--no-experts", action="store_true", help="quantise only the dense allow-list")
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--act-amax", type=float, default=GLOBAL)
    a = ap.parse_args(argv)
    search = (6.0, 5.0, 4.5, 4.0) if a.scale_search == "mse" else (FP4_MAX,)
    stats = convert(a.src, a.out, search, not a.no_experts, a.device, a.act_amax)
    print(json.dumps(stats))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
