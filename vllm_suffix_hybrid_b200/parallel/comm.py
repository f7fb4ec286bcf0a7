"""Collectives used by the tensor-parallel model.

``all_reduce`` routes by size and backend: the symmetric-memory NVLink
kernels (one-shot / two-shot, fused with residual-add + RMSNorm where the
caller asks for it) when the fused runtime is up, else NCCL (the baseline).
``vocab_parallel_argmax`` never gathers logits: every rank reduces its vocab
slice to (max, index) pairs and only those pairs cross the links.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import state

_FUSED = None  # parallel.symm.SymmComm when initialised


def set_fused(comm) -> None:
    global _FUSED
    _FUSED = comm


def fused():
    return _FUSED


def all_reduce(x: torch.Tensor) -> torch.Tensor:
    st = state.get()
    if st.tp == 1:
        return x
    if _FUSED is not None and _FUSED.can_all_reduce(x):
        return _FUSED.all_reduce(x)
    dist.all_reduce(x, group=st.group)
    return x


def all_reduce_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float) -> None:
    """x <- rms_norm(residual + allreduce(x)) * w, residual <- residual + allreduce(x)."""
    from .. import ops

    st = state.get()
    if st.tp > 1 and _FUSED is not None and _FUSED.can_all_reduce(x):
        _FUSED.all_reduce_add_rms_norm(x, residual, w, eps)
        return
    all_reduce(x)
    ops.fused_add_rms_norm(x, residual, w, eps)


def vocab_parallel_argmax(local_logits: torch.Tensor, vocab_offset: int, out: Optional[torch.Tensor] = None):
    """Global argmax over vocab-sharded logits [T, V/tp] without gathering them."""
    from .. import ops

    st = state.get()
    idx = ops.argmax(local_logits, out=None if st.tp > 1 else out)
    if st.tp == 1:
        return idx
    val = local_logits.gather(1, idx[:, None]).float()[:, 0]
    pair = torch.stack([val, (idx + vocab_offset).float()], dim=1)  # exact for ids < 2^24
    gathered = torch.empty(st.tp, *pair.shape, dtype=pair.dtype, device=pair.device)
    dist.all_gather_into_tensor(gathered, pair, group=st.group)
    vals, ids = gathered[..., 0], gathered[..., 1]
    best = vals.max(0, keepdim=True).values
    # Lowest global id among the maxima (first-occurrence semantics).
    cand = torch.where(vals == best, ids, torch.full_like(ids, float("inf")))
    res = cand.min(0).values.long()
    if out is not None:
        out.copy_(res)
        return out
    return res
