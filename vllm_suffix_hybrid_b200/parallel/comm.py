"""Collectives used by the tensor-parallel model.

``all_reduce`` routes by size and backend: the symmetric-memory NVLink
kernels (one-shot / two-shot, fused with residual-add + RMSNorm where the
caller asks for it) when the fused runtime is up, else NCCL (the baseline).
``vocab_parallel_argmax`` never gathers logits: every rank reduces its vocab
slice to (max, index) keys and only those keys cross the links -- in one
kernel over NVLink peer memory when the fused runtime is up (``_C.argmax_tp``),
else as an NCCL all-gather of (value, id) pairs (the baseline).
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


def _reduces(force: bool) -> bool:
    """Whether this process takes part in a world-wide reduction (TP, or EP when forced)."""
    st = state.get()
    return st.world > 1 and (st.tp > 1 or (force and st.ep > 1))


def can_push(tokens: int, hidden: int, like: torch.Tensor) -> bool:
    """Whether a row-parallel GEMM of this shape runs with the reduce-scatter in its epilogue."""
    f = _FUSED
    return (f is not None and getattr(f, "push_enabled", False) and state.get().tp > 1 and like.is_cuda
            and like.dtype == torch.bfloat16 and hidden == f.hidden and 0 < tokens <= f.max_tokens
            and like.shape[-1] % 64 == 0)


def push_gemm(x: torch.Tensor, w: torch.Tensor):
    return _FUSED.push_gemm(x, w)


def all_reduce(x: torch.Tensor, force: bool = False) -> torch.Tensor:
    """Sum over the ranks under TP (and under EP with force=True, for the MoE combine)."""
    if not isinstance(x, torch.Tensor):
        raise TypeError("a pushed row-parallel partial can only be finished by all_reduce_add_rms_norm")
    st = state.get()
    if not _reduces(force):
        return x
    if _FUSED is not None and _FUSED.can_all_reduce(x):
        return _FUSED.all_reduce(x)
    dist.all_reduce(x, group=st.group)
    return x


def partial_out(tokens: int, hidden: int, like: torch.Tensor, force: bool = False) -> Optional[torch.Tensor]:
    """Where a row-parallel GEMM (or the EP expert sum) should write its partial: the
    communicator's buffer when the fused comm runtime is on."""
    if _FUSED is not None and _reduces(force) and hidden == _FUSED.hidden and tokens <= _FUSED.max_tokens:
        return _FUSED.partial(tokens)
    return None


def all_reduce_add_rms_norm(x, residual: torch.Tensor, w: torch.Tensor, eps: float,
                            gather_residual: bool = False, prefetch: Optional[torch.Tensor] = None) -> torch.Tensor:
    """residual += allreduce(x); returns rms_norm(residual) * w (x may be reused as the output).

    x is a tensor partial, or the handle of a GEMM that pushed its rows to their owners: then each
    rank updates only the residual rows it owns (sequence-parallel residual) and every rank gets all
    normalised rows; gather_residual=True also brings every residual row up to date.  prefetch: the
    weight of the GEMM that reads the result, pulled into L2 by the fused kernel while the ranks wait.
    """
    from .. import ops

    if not isinstance(x, torch.Tensor):
        return x.comm.finish_push(x, residual, w, eps, gather_residual, prefetch)
    st = state.get()
    if st.tp > 1 and _FUSED is not None and _FUSED.can_all_reduce(x):
        return _FUSED.all_reduce_add_rms_norm(x, residual, w, eps, prefetch)
    if st.tp > 1:
        dist.all_reduce(x, group=st.group)
    ops.fused_add_rms_norm(x, residual, w, eps)
    return x


def vocab_parallel_argmax(local_logits: torch.Tensor, vocab_offset: int, out: Optional[torch.Tensor] = None):
    """Global argmax over vocab-sharded logits [T, V/tp] without gathering them."""
    from .. import ops

    st = state.get()
    if st.tp > 1 and _FUSED is not None and _FUSED.can_argmax(local_logits):
        return _FUSED.argmax(local_logits, vocab_offset, out)
    idx = ops.argmax(local_logits, out=None if st.tp > 1 else out)
    if st.tp == 1:
        return idx
    val = local_logits.gather(1, idx[:, None]).float()[:, 0]
    return vocab_parallel_best(val, idx, vocab_offset, out)


def vocab_parallel_best(val: torch.Tensor, idx: torch.Tensor, vocab_offset: int,
                        out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Global id of the best (value, local id) pair per row over the vocab shards (lowest id on ties)."""
    st = state.get()
    if st.tp == 1:
        if out is not None:
            out.copy_(idx)
            return out
        return idx
    pair = torch.stack([val.float(), (idx + vocab_offset).float()], dim=1)  # exact for ids < 2^24
    if pair.is_cuda:
        gathered = torch.empty(st.tp, *pair.shape, dtype=pair.dtype, device=pair.device)
        dist.all_gather_into_tensor(gathered, pair, group=st.group)
    else:
        parts = [torch.empty_like(pair) for _ in range(st.tp)]
        dist.all_gather(parts, pair, group=st.group)
        gathered = torch.stack(parts)
    vals, ids = gathered[..., 0], gathered[..., 1]
    best = vals.max(0, keepdim=True).values
    # Lowest global id among the maxima (first-occurrence semantics).
    cand = torch.where(vals == best, ids, torch.full_like(ids, float("inf")))
    res = cand.min(0).values.long()
    if out is not None:
        out.copy_(res)
        return out
    return res
