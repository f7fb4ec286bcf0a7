"""Tensor-parallel autograd collectives for training replays (Megatron-style).

copy_to_tp:     identity forward, all-reduce of the gradient (input of a column-parallel matmul)
reduce_from_tp: all-reduce forward, identity gradient (output of a row-parallel matmul)
gather_from_tp: all-gather along the last dimension forward, this rank's slice of the gradient
allreduce_grads: sum the gradients of replicated parameters over the TP ranks.
Without tensor parallelism every function is the identity.  Reference behaviour:
suffix_hybrid/mtp_tune/lora.py:1-40,151 (_CopyToTP, _ReduceFromTP, _GatherFromTP, allreduce_grads).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..parallel import state


def _group():
    st = state.get()
    return (st.group, st.tp) if st.tp > 1 else (None, 1)


class _Copy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        grp, tp = _group()
        if tp > 1:
            g = g.contiguous()
            dist.all_reduce(g, group=grp)
        return g


class _Reduce(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        grp, tp = _group()
        if tp > 1:
            x = x.contiguous().clone()
            dist.all_reduce(x, group=grp)
        return x

    @staticmethod
    def backward(ctx, g):
        return g


class _Gather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        grp, tp = _group()
        if tp == 1:
            return x
        parts = [torch.empty_like(x) for _ in range(tp)]
        dist.all_gather(parts, x.contiguous(), group=grp)
        ctx.width = x.shape[-1]
        return torch.cat(parts, -1)

    @staticmethod
    def backward(ctx, g):
        grp, tp = _group()
        if tp == 1:
            return g
        r = state.get().tp_rank
        return g[..., r * ctx.width:(r + 1) * ctx.width].contiguous()


def copy_to_tp(x):
    return _Copy.apply(x)


def reduce_from_tp(x):
    return _Reduce.apply(x)


def gather_from_tp(x):
    return _Gather.apply(x)


def allreduce_grads(params) -> None:
    grp, tp = _group()
    if tp == 1:
        return
    for p in params:
        if p.grad is not None:
            dist.all_reduce(p.grad, group=grp)


def broadcast_object(obj):
    """Rank 0's object on every TP rank (training plans are decided on rank 0)."""
    st = state.get()
    if st.tp == 1:
        return obj
    box = [obj]
    dist.broadcast_object_list(box, src=0, group=st.cpu_group if st.cpu_group is not None else st.group)
    return box[0]
