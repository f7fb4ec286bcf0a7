"""Process-group state: one process per GPU, torch.distributed over NCCL.

The tensor-parallel group is the whole world for the single-box layouts used
here (TP = N, or EP = N for the MoE configurations).  A CPU (gloo) group is
kept alongside for control-plane agreement (autotune decisions, barriers).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class ParallelState:
    rank: int = 0
    world: int = 1
    local_rank: int = 0
    tp: int = 1
    tp_rank: int = 0
    ep: int = 1
    ep_rank: int = 0
    dp: int = 1  # data-parallel attention: each rank serves its own requests (MoE experts shared by EP)
    dp_rank: int = 0
    group: Optional[object] = None  # device collectives
    cpu_group: Optional[object] = None  # control plane


_STATE = ParallelState()


def get() -> ParallelState:
    return _STATE


def init(tp: int = 1, ep: int = 1, backend: Optional[str] = None, timeout_s: int = 300, dp: int = 1) -> ParallelState:
    """Initialise from torchrun env vars (RANK/WORLD_SIZE/LOCAL_RANK/MASTER_*).

    dp = world (with tp = 1) selects data-parallel attention: every rank runs attention and dense layers for
    its own requests, and MoE layers exchange tokens with the other ranks (expert parallel over the world)."""
    global _STATE
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    group = dist.group.WORLD if world > 1 else None
    cpu_group = None
    if world > 1:
        cpu_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=timeout_s))
    if tp > 1 and tp != world:
        raise ValueError(f"tensor parallel size {tp} must equal the world size {world} on one box")
    if ep > 1 and ep != world:
        raise ValueError(f"expert parallel size {ep} must equal the world size {world} on one box")
    if dp > 1 and (dp != world or tp > 1):
        raise ValueError(f"data-parallel attention needs dp == world size ({world}) and tp == 1")
    _STATE = ParallelState(rank=rank, world=world, local_rank=local, tp=tp, tp_rank=rank if tp > 1 else 0, ep=ep,
                           ep_rank=rank if ep > 1 else 0, dp=dp, dp_rank=rank if dp > 1 else 0, group=group,
                           cpu_group=cpu_group)
    return _STATE


def shutdown() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()
