"""Dispatcher of the tcgen05 GEMM: y = x @ w^T for bf16 x [M, K], w [N, K].

Chooses per shape (cached) the orientation, the N-tile of the MMA and a
split-K factor so that the persistent grid fills the 148 SMs in whole waves:

* M <= 256: swap-AB -- the weight rows take the MMA's 128-row side and the
  tokens are the MMA N dimension (BN = 64/128/256), so a decode batch pays
  no padding to 128 rows;
* M > 256: activations on the 128-row side, weights tiled by BN = 128/256.

Split-K partials go to one fp32 workspace per device that grows on demand
and is reused by every call on that device's stream.
"""
from __future__ import annotations

import functools
import math
from typing import Dict, Optional

import torch

from . import native

NUM_SMS = 148
_WS: Dict[int, torch.Tensor] = {}


def _waves_eff(units: int, sms: int = NUM_SMS) -> float:
    return units / (math.ceil(units / sms) * sms)


@functools.lru_cache(maxsize=4096)
def plan(M: int, N: int, K: int):
    """(swap, bn, splits) for y[M, N] = x[M, K] w[N, K]^T.

    Split-K only when the tile grid is under one wave: its fp32 partials cost
    extra traffic and a reduce pass, so it must buy idle SMs.
    """
    kb = max(K // 64, 1)
    if M <= 256:
        bn = next(b for b in (64, 128, 256) if b >= M)
        tiles = math.ceil(N / 128) * math.ceil(M / bn)
        splits = 1
        while tiles * splits < NUM_SMS and kb // (splits * 2) >= 8 and splits < 8:
            splits *= 2
        return True, bn, splits
    bn = 256 if N > 8192 else 128
    tiles = math.ceil(M / 128) * math.ceil(N / bn)
    splits = 1
    # Split only grids that would leave most SMs idle: the fp32 partial
    # round trip costs more than a partly filled single wave.
    while tiles * splits < NUM_SMS // 3 and kb // (splits * 2) >= 16 and splits < 4:
        splits *= 2
    return False, bn, splits


def workspace(device: torch.device, numel: int) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WS.get(idx)
    if ws is None or ws.numel() < numel:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("GEMM split-K workspace must be sized before CUDA-graph capture (run once eagerly)")
        ws = torch.empty(max(numel, 1 << 20), dtype=torch.float32, device=device)
        _WS[idx] = ws
    return ws


def tcgen05_linear(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or x.shape[-1] % 64 != 0:
        raise ValueError(f"tcgen05 GEMM needs bf16 operands with K % 64 == 0 (got {x.dtype}, K={x.shape[-1]})")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1 or (x2.stride(0) * 2) % 16 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    M, K = x2.shape
    N = w.shape[0]
    y = out.view(M, N) if out is not None else torch.empty(M, N, dtype=x.dtype, device=x.device)
    if M == 0:
        return y.view(*lead, N)
    swap, bn, splits = plan(M, N, K)
    ws = workspace(x.device, splits * M * N) if splits > 1 else None
    native().gemm_bf16(y, x2, w, swap, bn, splits, ws)
    return y.view(*lead, N)
