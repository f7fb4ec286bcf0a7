"""Expert parallelism: each of the N ranks holds E/N routed experts.

Layout of the reference's EP (reference: suffix_hybrid/kernels/nvfp4_moe.py:78-84,449-457 and
docs/dsv41-comms.md:54-58): every rank sees every token (attention is replicated or tensor
parallel), the router runs on every rank, each rank computes only the (token, expert) pairs of its
local experts -- expert ids are rebased by ``ep_rank * E_local`` and pairs routed elsewhere are
skipped by the align kernel -- and one all-reduce sums the ranks' partial outputs.  The partial is
written straight into the communicator's buffer, so the combine is this framework's NVLink
all-reduce kernel (or NCCL with ``comm=nccl``).
"""
from __future__ import annotations

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
    else:
        out = ops.moe_experts(x, ids_l, w_l, moe.w13, moe.w2, moe.E_local, moe.F, out=out)
    return comm.all_reduce(out, force=True)
