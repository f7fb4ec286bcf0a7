"""Model families: dense Llama, Qwen3-Next hybrid GDN/MoE, DeepSeek-V3.2 / Kimi-K2 MLA MoE."""
from __future__ import annotations


def build_model(cfg, device, seed: int = 0, with_draft: bool = True):
    """(target, draft head or None) for a ModelConfig."""
    if cfg.arch == "llama":
        from .llama import DraftHead, LlamaModel

        m = LlamaModel(cfg, device, seed)
        d = DraftHead(cfg, m, device, style="mtp" if cfg.draft == "mtp" else "eagle") if with_draft else None
        return m, d
    if cfg.arch == "qwen3_next":
        from .qwen3_next import build

        return build(cfg, device, seed, with_draft)
    if cfg.arch in ("deepseek_v32", "kimi_k2"):
        from .deepseek import build

        return build(cfg, device, seed, with_draft)
    raise ValueError(f"unknown architecture {cfg.arch}")
