"""Expert parallelism: each of the N ranks holds E/N routed experts.

Two layouts.  With replicated (or tensor-parallel) attention every rank sees every token:
`dispatch_combine` below.  With data-parallel attention (state.dp > 1) every rank holds different
tokens: `dp_dispatch_combine` sends each token row only to the ranks that host its experts and returns
the expert outputs to the owner, with P2P stores from the kernels of ``parallel/ep_a2a.py`` (CUDA), or
gathers all ranks' tokens and routes, runs this rank's experts over them and reduce-scatters the partial
outputs back (NCCL / gloo, ``SH_EP_A2A=0``); the engine pads every rank to the same token count per call.

Layout of the reference's EP (reference: suffix_hybrid/kernels/nvfp4_moe.py:78-84,449-457 and
docs/dsv41-comms.md:54-58): every rank sees every token (attention is replicated or tensor
parallel), the router runs on every rank, each rank computes only the (token, expert) pairs of its
local experts -- expert ids are rebased by ``ep_rank * E_local`` and pairs routed elsewhere are
skipped by the align kernel -- and one all-reduce sums the ranks' partial outputs.  The partial is
written straight into the communicator's buffer, so the combine is this framework's NVLink
all-reduce kernel (or NCCL with ``comm=nccl``).
"""
from __future__ import annotations

import os

import torch

from .. import ops
from . import comm, state


def local_routes(ids: torch.Tensor, w: torch.Tensor, e0: int, e_local: int):
    """(ids rebased to this rank's experts, -1 elsewhere; weights, 0 elsewhere)."""
    mine = (ids >= e0) & (ids < e0 + e_local)
    return torch.where(mine, ids - e0, torch.full_like(ids, -1)), torch.where(mine, w, torch.zeros_like(w))


def dispatch_combine(moe, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """sum over all experts of w * FFN_e(x), with this rank's experts local and one all-reduce."""
    st = state.get()
    T, H = x.shape
    ids_l, w_l = local_routes(ids, w, st.ep_rank * moe.E_local, moe.E_local)
    out = comm.partial_out(T, H, x, force=True)
    if moe.fp4 is not None:
        out = ops.moe_experts_nvfp4(x, ids_l, w_l, moe.fp4[0], moe.fp4[1], moe.E_local, moe.F, out=out)
    elif getattr(moe, "fp8", None) is not None:
        out = ops.moe_experts_mxfp8(x, ids_l, w_l, moe.fp8[0], moe.fp8[1], moe.E_local, moe.F, out=out)
    else:
        out = ops.moe_experts(x, ids_l, w_l, moe.w13, moe.w2, moe.E_local, moe.F, out=out)
    return comm.all_reduce(out, force=True)


def _all_gather(x: torch.Tensor) -> torch.Tensor:
    import torch.distributed as dist

    st = state.get()
    x = x.contiguous()
    if x.is_cuda:
        out = torch.empty((st.world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x, group=st.group)
        return out
    parts = [torch.empty_like(x) for _ in range(st.world)]
    dist.all_gather(parts, x, group=st.group)
    return torch.cat(parts, 0)


def _reduce_scatter(y: torch.Tensor) -> torch.Tensor:
    import torch.distributed as dist

    st = state.get()
    T = y.shape[0] // st.world
    if y.is_cuda:
        out = torch.empty((T,) + tuple(y.shape[1:]), dtype=y.dtype, device=y.device)
        dist.reduce_scatter_tensor(out, y.contiguous(), group=st.group)
        return out
    y = y.contiguous().clone()
    dist.all_reduce(y, group=st.group)  # gloo has no reduce-scatter
    return y[st.rank * T:(st.rank + 1) * T].contiguous()


def _experts(moe, xs: torch.Tensor, ids_l: torch.Tensor, w_l: torch.Tensor) -> torch.Tensor:
    if moe.fp4 is not None:
        return ops.moe_experts_nvfp4(xs, ids_l, w_l, moe.fp4[0], moe.fp4[1], moe.E_local, moe.F)
    if getattr(moe, "fp8", None) is not None:
        return ops.moe_experts_mxfp8(xs, ids_l, w_l, moe.fp8[0], moe.fp8[1], moe.E_local, moe.F)
    return ops.moe_experts(xs, ids_l, w_l, moe.w13, moe.w2, moe.E_local, moe.F)


A2A_MAX_TOKENS = int(os.environ.get("SH_EP_A2A_MAX_TOKENS", "4096"))


def a2a_enabled(x: torch.Tensor) -> bool:
    """Device all-to-all over NVLink peer memory (SH_EP_A2A=0: NCCL all-gather / reduce-scatter).  The
    decision depends only on values equal on every rank (device kind, world, T)."""
    st = state.get()
    return (x.is_cuda and st.world > 1 and os.environ.get("SH_EP_A2A", "1") != "0"
            and x.shape[0] <= A2A_MAX_TOKENS)


def _quant_dispatch(moe, x: torch.Tensor) -> bool:
    return (moe.fp4 is not None and ops.nvfp4_act_mode() == "fp4" and x.shape[1] % 256 == 0
            and os.environ.get("SH_EP_A2A_FP4", "1") != "0")


def _a2a_experts_combine(moe, comm, quant: bool, rows, ids_l: torch.Tensor, w_l: torch.Tensor,
                         ids: torch.Tensor) -> torch.Tensor:
    """Experts over the received rows, then the combine.  By default the experts' weighted per-token sum
    stores its rows straight into the owners' return rows (one launch, no local output; bit-identical);
    SH_EP_COMBINE_PUSH=0 writes the local output and lets ep_combine copy it."""
    if os.environ.get("SH_EP_COMBINE_PUSH", "1") == "0":
        if quant:  # NVFP4 rows: the W4A4 experts gather the received codes directly
            y = ops.moe_experts_nvfp4(None, ids_l, w_l, moe.fp4[0], moe.fp4[1], moe.E_local, moe.F, prequant=rows)
        else:
            y = _experts(moe, rows, ids_l, w_l)
        return comm.combine(y, ids)
    T = ids.shape[0]

    def push(ys, sorted_pos):
        comm.combine_push(ys, sorted_pos, w_l, ids_l, T)

    if quant:
        ops.moe_experts_nvfp4(None, ids_l, w_l, moe.fp4[0], moe.fp4[1], moe.E_local, moe.F, prequant=rows, push=push)
    elif moe.fp4 is not None:
        ops.moe_experts_nvfp4(rows, ids_l, w_l, moe.fp4[0], moe.fp4[1], moe.E_local, moe.F, push=push)
    elif getattr(moe, "fp8", None) is not None:
        ops.moe_experts_mxfp8(rows, ids_l, w_l, moe.fp8[0], moe.fp8[1], moe.E_local, moe.F, push=push)
    else:
        ops.moe_experts(rows, ids_l, w_l, moe.w13, moe.w2, moe.E_local, moe.F, push=push)
    return comm.combine_sum(ids)


def dp_route_dispatch_combine(moe, x: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
    """dp_dispatch_combine with the router top-k run inside the dispatch kernel (CUDA all-to-all only):
    logits [T, E] -> [T, H].  Bit-identical to ops.moe_route followed by dp_dispatch_combine."""
    from . import ep_a2a

    quant = _quant_dispatch(moe, x)
    comm = ep_a2a.get(x.shape[1], A2A_MAX_TOKENS, moe.k, moe.E_local, quant)
    rows, ids_l, w_l, ids, _ = comm.dispatch_routed(x, logits, **moe.route_args())
    return _a2a_experts_combine(moe, comm, quant, rows, ids_l, w_l, ids)


def dp_dispatch_combine(moe, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Data-parallel attention: every rank's tokens through this rank's experts; each rank keeps its own rows.

    x [T, H] (T equal on every rank), ids / w [T, k] from the local router; returns [T, H]."""
    st = state.get()
    if a2a_enabled(x):
        from . import ep_a2a

        quant = _quant_dispatch(moe, x)
        comm = ep_a2a.get(x.shape[1], A2A_MAX_TOKENS, ids.shape[1], moe.E_local, quant)
        rows, ids_l, w_l = comm.dispatch(x, ids, w)
        return _a2a_experts_combine(moe, comm, quant, rows, ids_l, w_l, ids)
    xs = _all_gather(x)
    ids_a = _all_gather(ids)
    w_a = _all_gather(w)
    ids_l, w_l = local_routes(ids_a, w_a, st.ep_rank * moe.E_local, moe.E_local)
    return _reduce_scatter(_experts(moe, xs, ids_l, w_l))
