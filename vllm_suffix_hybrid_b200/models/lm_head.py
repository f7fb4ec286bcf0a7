"""NVFP4-screened LM head for greedy decoding (SUFFIX_NVFP4_LMHEAD=1, default off).

The vocab projection is the largest single weight read of a decode step on NVFP4 checkpoints that keep
the head in bf16.  For batches of at most SUFFIX_NVFP4_LMHEAD_MAX_M rows (default 64) the head is
screened with the block-scaled W4A4 tcgen05 GEMM (weights quantised once at install, activations
quantised per token), the SUFFIX_NVFP4_LMHEAD_RESCORE best candidates per row (default 64) are
re-scored exactly in fp32 from the resident bf16 rows, and the argmax is taken over those exact values.
Greedy picks therefore see exact logits whenever the true argmax is among the screened candidates;
the W4A4 noise only reaches the tail.  Larger batches (the prefill, wide verify windows) use the bf16
head.  Under tensor parallelism each rank screens its vocab shard and the (value, id) pairs are combined
by the vocab-parallel argmax.  Every step is static-shape, so it is captured inside the decode graphs.

Reference behaviour: suffix_hybrid/kernels/nvfp4_lm_head.py:1-60 (load-time NVFP4 quantisation of the
head, dynamic per-call activation scale, W4A4 screen, top-RESCORE exact bf16 re-score, M cap).
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from .. import ops
from ..ops import reference as ref

MAX_M = 64
RESCORE = 64


def enabled() -> bool:
    return os.environ.get("SUFFIX_NVFP4_LMHEAD", "").strip() == "1"


def _env_int(name: str, default: int, lo: int, hi: int) -> int:
    raw = os.environ.get(name, "").strip()
    if not raw:
        return default
    if not raw.isdigit() or not lo <= int(raw) <= hi:
        raise ValueError(f"{name}={raw!r}: need an integer in {lo}..{hi}")
    return int(raw)


class ScreenedHead:
    """NVFP4 copy of a bf16 head weight [V_local, H] plus the exact re-score of screened candidates."""

    def __init__(self, weight: torch.Tensor):
        self.weight = weight  # bf16, stays resident (re-score rows, tied embeddings)
        self.max_m = _env_int("SUFFIX_NVFP4_LMHEAD_MAX_M", MAX_M, 1, 4096)
        self.rescore = min(_env_int("SUFFIX_NVFP4_LMHEAD_RESCORE", RESCORE, 1, 4096), weight.shape[0])
        if weight.is_cuda:
            self.packed, self.scales, self.gscale = ops.nvfp4_quantize(weight)
            self.w_sf = ops.nvfp4_scale_tiles(self.scales)
        else:
            g = ref.nvfp4_global_scale(weight)
            self.packed, self.scales = ref.nvfp4_quantize(weight, g)
            self.gscale, self.w_sf = g, None

    def applies(self, x: torch.Tensor) -> bool:
        return x.dim() == 2 and x.shape[0] <= self.max_m and x.dtype == torch.bfloat16 and x.shape[1] % 64 == 0

    def screen(self, x: torch.Tensor) -> torch.Tensor:
        """Approximate logits [M, V_local] (W4A4)."""
        if x.is_cuda:
            return ops.nvfp4_linear_w4a4(x, self.packed, self.w_sf, self.scales, self.gscale)
        return ref.nvfp4_w4a4_linear(x, self.packed, self.scales, self.gscale)

    def best(self, x: torch.Tensor):
        """(exact value fp32 [M], local id [M]) of the best screened candidate per row."""
        approx = self.screen(x)
        top = approx.float().topk(self.rescore, dim=-1).indices  # [M, R]
        rows = self.weight.index_select(0, top.reshape(-1)).view(x.shape[0], self.rescore, -1)
        # fp32 dot products rounded to the head's output dtype, as the bf16 head's logits are
        exact = torch.bmm(rows.float(), x.float().unsqueeze(-1)).squeeze(-1).to(self.weight.dtype).float()
        # lowest vocab id among the maxima (first-occurrence semantics of the bf16 head's argmax)
        mx = exact.max(-1, keepdim=True).values
        ids = torch.where(exact == mx, top, torch.full_like(top, torch.iinfo(torch.long).max)).min(-1).values
        return mx[:, 0], ids


def install(model) -> Optional[ScreenedHead]:
    """Attach a screened head to a model whose `lm_head` holds a bf16 weight (after weights are loaded)."""
    head = getattr(model, "lm_head", None)
    if head is None or isinstance(getattr(type(head), "weight", None), property):
        return None  # quantised heads decode on demand: nothing to screen
    w = getattr(head, "weight", None)
    if w is None or w.dtype != torch.bfloat16:
        return None
    model.lm_screen = ScreenedHead(w)
    return model.lm_screen
