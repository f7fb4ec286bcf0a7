"""Dispatcher of the tcgen05 GEMMs: y = x @ w^T for bf16 x [M, K], w [N, K].

Three kernel families, all on the 5th-generation tensor cores:

* ``tc``   -- one CTA per 128-row tile (csrc/kernels/gemm_tcgen05.cu);
* ``pair`` -- a CTA pair (cta_group::2) per 256-row tile, same file;
* ``sk``   -- stream-K on CTA pairs with the weights on the MMA M side and
  every token of the call in one wide N tile (csrc/kernels/gemm_streamk.cu):
  each weight byte crosses HBM once and all SMs get equal MMA work.

A configuration is ``Cfg(kind, swap, bn, splits, clusters)``:

* tc / pair: swap puts the weight rows on the MMA M side (tokens become N),
  bn is the MMA N tile (tc 64/128/256, pair 128/192/256) and splits the
  split-K factor (fp32 partials + a deterministic reduce pass);
* sk: bn is the MMA N per instruction (64/128/192/256), splits the number of
  MMAs per 16-wide k-step (1 or 2; tokens per tile = bn * splits) and
  clusters the number of CTA pairs sharing the iteration space;
* lib: cuBLAS (torch.matmul), only a candidate when SH_GEMM_LIB=1.

Every new (M, N, K) is autotuned once, on its first eager call: the
candidates are timed on the device with a cold L2 and the fastest is kept
for the process (SH_GEMM_TUNE=0 uses the static heuristic;
SH_GEMM_TUNE_FILE=path loads and saves the choices as JSON, which pins them
across runs and across processes of a multi-GPU job).  Calls during
CUDA-graph capture never tune: they use the recorded choice or the
heuristic.

Batch-invariant mode (SH_BATCH_INVARIANT=1): no autotuning; every call with
M <= 256 runs the one-CTA swap-AB kernel with a 64-token N tile and every
larger call the CTA-pair kernel, with the split-K factor a function of
(N, K) alone, so a token's output does not depend on how many other tokens
share the call (a k+1-token verify window gives the same logits as plain
decoding).  Stream-K pieces depend on the tile count, so sk is not used in
that mode.

Split-K partials, stream-K partial slots and stream-K arrival counters live
in per-device buffers that grow on demand and are reused by every call on
that device's stream (one GEMM at a time per device).
"""
from __future__ import annotations

import functools
import json
import math
import os
from typing import Dict, NamedTuple, Optional, Tuple

import torch

from . import native

NUM_SMS = 148
_WS: Dict[int, torch.Tensor] = {}
_SK_WS: Dict[int, torch.Tensor] = {}
_SK_CNT: Dict[int, torch.Tensor] = {}
_RETIRED: list = []


class Cfg(NamedTuple):
    kind: str        # "tc" | "pair" | "sk" | "lib"
    swap: bool = False
    bn: int = 0
    splits: int = 1
    clusters: int = 0


LIB = Cfg("lib")
SK_SHAPES = ((64, 1), (128, 1), (192, 1), (256, 1), (192, 2), (256, 2))  # (MMA N, MMAs per k-step)


def sk_tokens(bn: int, nsub: int) -> int:
    return bn * nsub


@functools.lru_cache(maxsize=64)
def sk_max_clusters(bn: int, nsub: int) -> int:
    return int(native().gemm_sk_max_clusters(bn, nsub)) or NUM_SMS // 2


@functools.lru_cache(maxsize=4096)
def heuristic(M: int, N: int, K: int) -> Cfg:
    """Configuration without measurement.

    Up to 512 tokens: stream-K with every token in one tile (the narrowest
    tile that holds them) on all co-resident CTA pairs.  Larger M is bound by
    the L2 -> SM operand stream, where the CTA pair's 256 x 256 tile moves the
    fewest bytes per MAC.
    """
    if M <= 512 and N % 8 == 0 and not batch_invariant():
        bn, nsub = next((b, u) for b, u in SK_SHAPES if sk_tokens(b, u) >= M)
        return Cfg("sk", True, bn, nsub, NUM_SMS // 2)
    kb = max(K // 64, 1)
    if M <= 256:
        bn = next(b for b in (64, 128, 256) if b >= M)
        tiles = math.ceil(N / 128) * math.ceil(M / bn)
        splits = 1
        while tiles * splits * 2 <= NUM_SMS and kb // (splits * 2) >= 8 and splits < 8:
            splits *= 2
        return Cfg("tc", True, bn, splits)
    tiles = math.ceil(M / 256) * math.ceil(N / 256)
    splits = 1
    while tiles * splits < NUM_SMS // 4 and kb // (splits * 2) >= 16 and splits < 4:
        splits *= 2
    return Cfg("pair", False, 256, splits)


def batch_invariant() -> bool:
    return os.environ.get("SH_BATCH_INVARIANT", "0") == "1"


@functools.lru_cache(maxsize=4096)
def invariant_splits(N: int, K: int) -> int:
    """Split-K factor of (N, K) used for every M in batch-invariant mode (the decode-size choice)."""
    kb = max(K // 64, 1)
    tiles = math.ceil(N / 128)
    splits = 1
    while tiles * splits * 2 <= NUM_SMS and kb // (splits * 2) >= 8 and splits < 8:
        splits *= 2
    return splits


def candidates(M: int, N: int, K: int, splits_only: Optional[int] = None):
    kb = max(K // 64, 1)
    out = [LIB] if os.environ.get("SH_GEMM_LIB", "0") == "1" and splits_only is None else []
    if splits_only is None and N % 8 == 0 and os.environ.get("SH_GEMM_SK", "1") != "0":
        tiles_w = math.ceil(N / 256)
        fits = [(b, u) for b, u in SK_SHAPES if sk_tokens(b, u) >= M]
        # the narrowest single tile over all tokens, and narrower tiles that split the tokens
        shapes = fits[:1] + [(b, u) for b, u in SK_SHAPES if sk_tokens(b, u) < M and sk_tokens(b, u) >= M / 4]
        for b, u in shapes:
            tiles = tiles_w * math.ceil(M / sk_tokens(b, u))
            gmax = sk_max_clusters(b, u)
            for g in sorted({gmax, min(gmax, tiles), min(gmax, 2 * tiles)}):
                out.append(Cfg("sk", True, b, u, g))
    for pair in (False, True):
        for swap in (False, True):
            for bn in ((128, 192, 256) if pair else (64, 128, 256)):
                if bn >= 2 * max(M if swap else N, 64) and bn > 64:
                    continue  # tile far wider than the operand
                for splits in ((splits_only,) if splits_only else (1, 2, 4)):
                    if splits_only is None and splits > 1 and kb // splits < 4:
                        continue
                    out.append(Cfg("pair" if pair else "tc", swap, bn, splits))
    return out


_CHOICE: Dict[Tuple[int, int, int], Cfg] = {}
_FLUSH: Dict[int, torch.Tensor] = {}
_LOADED = [False]


def _tune_file() -> Optional[str]:
    return os.environ.get("SH_GEMM_TUNE_FILE") or None


def _load():
    if _LOADED[0]:
        return
    _LOADED[0] = True
    f = _tune_file()
    if f and os.path.exists(f):
        with open(f) as fh:
            for key, val in json.load(fh).items():
                M, N, K = (int(v) for v in key.split(","))
                if isinstance(val, list) and len(val) == 5 and isinstance(val[0], str):
                    _CHOICE[(M, N, K)] = Cfg(val[0], bool(val[1]), int(val[2]), int(val[3]), int(val[4]))


def _save():
    f = _tune_file()
    if not f:
        return
    data = {f"{M},{N},{K}": list(v) for (M, N, K), v in sorted(_CHOICE.items())}
    tmp = f + ".tmp"
    with open(tmp, "w") as fh:
        json.dump(data, fh, indent=0)
    os.replace(tmp, f)


def _autotune(x2: torch.Tensor, w: torch.Tensor, y: torch.Tensor, splits_only: Optional[int] = None) -> Cfg:
    M, K = x2.shape
    N = w.shape[0]
    dev = x2.device
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    flush = _FLUSH.get(idx)
    if flush is None:
        flush = _FLUSH[idx] = torch.empty(160 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    cands = candidates(M, N, K, splits_only)
    times = []
    for cfg in cands:
        run = _runner(cfg, x2, w, y)
        try:
            run()  # first launch: no timing
        except RuntimeError:  # a configuration this shape cannot use (alignment, size)
            times.append(float("inf"))
            continue
        t = float("inf")
        for _ in range(2):
            flush.zero_()  # cold L2, and keeps the GPU busy while the timed launch is enqueued
            torch.cuda._sleep(50_000)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            run()
            e.record()
            e.synchronize()
            t = min(t, s.elapsed_time(e))
        times.append(t)
    times = _agree(times)
    return cands[min(range(len(cands)), key=times.__getitem__)]


def _sk_buffers(device: torch.device, ws_floats: int, counters: int):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws, cnt = _SK_WS.get(idx), _SK_CNT.get(idx)
    if ws is None or ws.numel() < ws_floats or cnt is None or cnt.numel() < counters:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("stream-K GEMM buffers must be sized before CUDA-graph capture (run once eagerly)")
        # Replaced buffers stay alive: CUDA graphs captured earlier still point at them.
        if ws is None or ws.numel() < ws_floats:
            _RETIRED.append(ws)
            ws = _SK_WS[idx] = torch.empty(max(ws_floats, 1 << 20), dtype=torch.float32, device=device)
        if cnt is None or cnt.numel() < counters:
            _RETIRED.append(cnt)
            cnt = _SK_CNT[idx] = torch.zeros(max(counters, 4096), dtype=torch.int32, device=device)
    return ws, cnt


def _runner(cfg: Cfg, x2, w, y):
    if cfg.kind == "lib":
        return lambda: torch.matmul(x2, w.t(), out=y)
    M, N = x2.shape[0], w.shape[0]
    if cfg.kind == "sk":
        nt = cfg.bn * cfg.splits
        tiles = math.ceil(N / 256) * math.ceil(M / nt)
        ws, cnt = _sk_buffers(x2.device, cfg.clusters * 4 * nt * 128, 2 * tiles)
        return lambda: native().gemm_bf16_sk(y, x2, w, cfg.bn, cfg.splits, cfg.clusters, ws, cnt)
    ws = workspace(x2.device, cfg.splits * M * N) if cfg.splits > 1 else None
    return lambda: native().gemm_bf16(y, x2, w, cfg.swap, cfg.bn, cfg.splits, ws, None, cfg.kind == "pair")


def _agree(times):
    """Sum the candidates' times over the tensor-parallel ranks so every rank picks the same configuration.

    Ranks that chose differently would run different kernels per layer and
    wait for each other at every all-reduce.  Every rank autotunes the same
    shapes in the same order (the TP-sharded model is identical per rank).
    """
    try:
        import torch.distributed as dist

        from ..parallel import state

        st = state.get()
        if not dist.is_initialized() or st.tp <= 1 or st.tp != st.world or st.cpu_group is None:
            return times
        t = torch.tensor(times, dtype=torch.float64)
        dist.all_reduce(t, group=st.cpu_group)
        return t.tolist()
    except Exception:
        return times


def plan(M: int, N: int, K: int, x2: Optional[torch.Tensor] = None, w: Optional[torch.Tensor] = None,
         y: Optional[torch.Tensor] = None) -> Cfg:
    """Configuration for y[M, N] = x[M, K] w[N, K]^T (see the module docstring)."""
    _load()
    inv = batch_invariant()
    key = (M, N, K) if not inv else (-M, N, K)
    got = _CHOICE.get(key)
    if got is not None:
        return got
    if inv:
        # One kernel family per M range and split-K from (N, K) alone: nothing about a row's
        # arithmetic depends on how many rows share the call.
        fixed = invariant_splits(N, K)
        got = Cfg("tc", True, 64, fixed) if M <= 256 else Cfg("pair", False, 256, fixed)
        _CHOICE[key] = got
        return got
    if (x2 is None or os.environ.get("SH_GEMM_TUNE", "1") == "0" or torch.cuda.is_current_stream_capturing()):
        return heuristic(M, N, K)
    got = _autotune(x2, w, y, None)
    _CHOICE[key] = got
    if not inv:
        _save()
    return got


_PUSH: Dict[Tuple[int, int, int], Tuple[bool, int]] = {}


def plan_push(x2: torch.Tensor, w: torch.Tensor) -> Tuple[bool, int]:
    """(pair, bn) of a push (reduce-scatter epilogue) GEMM: tokens on the M side, no split-K.

    Timed on the same tile configurations with the local epilogue (a push run cannot be timed
    alone: it counts arrivals at the peers); the choice is agreed across ranks like every plan.
    """
    M, K = x2.shape
    N = w.shape[0]
    key = (M, N, K)
    got = _PUSH.get(key)
    if got is not None:
        return got
    if torch.cuda.is_current_stream_capturing() or os.environ.get("SH_GEMM_TUNE", "1") == "0":
        return (M > 128, 256 if M > 128 else 128)
    y = torch.empty(M, N, dtype=x2.dtype, device=x2.device)
    cands = [Cfg("tc", False, bn, 1) for bn in (64, 128, 256)] + [Cfg("pair", False, bn, 1) for bn in (128, 192, 256)]
    dev = x2.device
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    flush = _FLUSH.get(idx)
    if flush is None:
        flush = _FLUSH[idx] = torch.empty(160 << 20, dtype=torch.uint8, device=dev)
    times = []
    for cfg in cands:
        run = _runner(cfg, x2, w, y)
        run()
        t = float("inf")
        for _ in range(2):
            flush.zero_()
            torch.cuda._sleep(50_000)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            run()
            e.record()
            e.synchronize()
            t = min(t, s.elapsed_time(e))
        times.append(t)
    times = _agree(times)
    best = cands[min(range(len(cands)), key=times.__getitem__)]
    _PUSH[key] = (best.kind == "pair", best.bn)
    return _PUSH[key]


def choice_summary() -> dict:
    """How many tuned shapes run which kernel family (for benchmark reports)."""
    names = {"tc": "tcgen05_one_cta", "pair": "tcgen05_pair", "sk": "tcgen05_streamk", "lib": "cublas"}
    out = {v: 0 for v in names.values()}
    for cfg in _CHOICE.values():
        out[names[cfg.kind]] += 1
    return out


def workspace(device: torch.device, numel: int) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WS.get(idx)
    if ws is None or ws.numel() < numel:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("GEMM split-K workspace must be sized before CUDA-graph capture (run once eagerly)")
        _RETIRED.append(ws)  # graphs captured earlier may still point at it
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
    cfg = plan(M, N, K, x2, w, y)
    _runner(cfg, x2, w, y)()
    return y.view(*lead, N)
