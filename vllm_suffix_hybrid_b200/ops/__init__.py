"""Kernel entry points.

On a CUDA device every op runs the in-tree sm_100a kernel from ``_C``; a
missing or stale extension is an error, never a silent PyTorch fallback.  On
the CPU (the toy configuration and the CPU test suite) the ops run their
plain-PyTorch statement from :mod:`.reference`.
"""
from __future__ import annotations

import importlib
import os

import torch

from . import reference as ref

_C = None
_C_ERR = None


class _Counting:
    """Proxy counting kernel launches issued through the extension."""

    def __init__(self, mod):
        self._mod = mod
        self.count = 0
        self.by_name = {}

    def __getattr__(self, name):
        fn = getattr(self._mod, name)

        def wrapped(*a, **kw):
            self.count += 1
            self.by_name[name] = self.by_name.get(name, 0) + 1
            return fn(*a, **kw)

        return wrapped


_COUNTER = None


def count_launches(enable: bool):
    """Start (True) or stop (False) counting; returns the counter."""
    global _COUNTER
    c = _COUNTER
    _COUNTER = _Counting(native()) if enable else None
    return _COUNTER if enable else c


def native():
    """The compiled kernel module; raises if it cannot be loaded."""
    global _C, _C_ERR
    if _COUNTER is not None:
        return _COUNTER
    if _C is None:
        try:
            _C = importlib.import_module("vllm_suffix_hybrid_b200._C")
        except Exception as e:  # pragma: no cover - exercised on hosts without the build
            _C_ERR = e
            raise RuntimeError(
                "vllm_suffix_hybrid_b200._C (sm_100a kernels) is not built or failed to load: "
                f"{e!r}. Run `python setup.py build_ext --inplace` on this source tree."
            ) from e
    return _C


def _cuda(t: torch.Tensor) -> bool:
    return t.is_cuda


# ----------------------------------------------------------------------------- norms
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    if not _cuda(x):
        r = ref.rms_norm(x, w, eps)
        if out is not None:
            out.copy_(r)
            return out
        return r
    if out is None:
        out = torch.empty_like(x)
    native().rms_norm(out.view(-1, x.shape[-1]), x.view(-1, x.shape[-1]), w, eps)
    return out


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float) -> None:
    """residual += x; x = rms_norm(residual) * w   (both in place)."""
    if not _cuda(x):
        ref.fused_add_rms_norm(x, residual, w, eps)
        return
    native().fused_add_rms_norm(x, residual, w, eps)


# ----------------------------------------------------------------------------- rotary + cache
def rope_kv_write(qkv, positions, cos_sin, k_cache, v_cache, slot_mapping, hq, hk, d, rot=None) -> None:
    rot = d if rot is None else rot
    if not _cuda(qkv):
        ref.rope_kv_write(qkv, positions, cos_sin, k_cache, v_cache, slot_mapping, hq, hk, d, rot)
        return
    native().rope_kv_write(qkv, positions, cos_sin, k_cache, v_cache, slot_mapping, hq, hk, d, rot)


# ----------------------------------------------------------------------------- attention
def plan_attention_tiles(q_lens, group: int, rows: int = 64):
    """(tile_req, tile_row0) int32 lists: one entry per 64-row query tile."""
    req, row0 = [], []
    for b, ql in enumerate(q_lens):
        n = int(ql) * group
        for r in range(0, n, rows):
            req.append(b)
            row0.append(r)
    return req, row0


_ATTN_WS = {}


def attention_splits(num_tiles: int, kv_heads: int, max_pages: int, sms: int = 148) -> int:
    """KV splits per request so the grid covers ~4 waves of SMs (1..16)."""
    units = max(num_tiles * kv_heads, 1)
    want = -(-4 * sms // units)
    return int(max(1, min(16, want, max(1, max_pages // 2))))


def _attn_workspace(device, n_o: int, n_ml: int):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _ATTN_WS.get(idx)
    if ws is None or ws[0].numel() < n_o or ws[1].numel() < n_ml:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("attention split-KV workspace must be sized before CUDA-graph capture")
        ws = (torch.empty(max(n_o, 1 << 16), dtype=torch.float32, device=device),
              torch.empty(max(n_ml, 1 << 12), dtype=torch.float32, device=device))
        _ATTN_WS[idx] = ws
    return ws


def paged_attention(out, q, k_cache, v_cache, block_tables, seq_lens, q_start, tile_req, tile_row0, hq, scale,
                    nsplit: int = 1, max_rows: int = 64):
    """out[T, hq*D] <- attention of q (rows of the QKV buffer) over the paged cache."""
    if not _cuda(q):
        d = k_cache.shape[3]
        t = q.shape[0]
        qv = q[:, : hq * d].reshape(t, hq, d)
        out.view(t, hq, d).copy_(ref.paged_attention(qv, k_cache, v_cache, block_tables, seq_lens, q_start, hq, scale))
        return out
    if nsplit > 1:
        d = k_cache.shape[3]
        n = q.shape[0] * hq * nsplit
        po, pml = _attn_workspace(q.device, n * d, n * 2)
        native().paged_attention(out, q, k_cache, v_cache, block_tables, seq_lens, q_start, tile_req, tile_row0, hq,
                                 scale, nsplit, po, pml, None, max_rows)
    else:
        native().paged_attention(out, q, k_cache, v_cache, block_tables, seq_lens, q_start, tile_req, tile_row0, hq,
                                 scale, 1, None, None, None, max_rows)
    return out


# ----------------------------------------------------------------------------- activations / gather
def silu_mul(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if not _cuda(x):
        r = ref.silu_mul(x)
        if out is not None:
            out.copy_(r)
            return out
        return r
    if out is None:
        out = torch.empty(*x.shape[:-1], x.shape[-1] // 2, dtype=x.dtype, device=x.device)
    native().silu_mul(out, x)
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if not _cuda(table):
        r = table[ids.clamp(0, table.shape[0] - 1)]
        if out is not None:
            out.copy_(r)
            return out
        return r
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    native().embedding(out, ids.reshape(-1), table)
    return out


# ----------------------------------------------------------------------------- sampling / verify
def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if not _cuda(logits):
        r = logits.float().argmax(-1)
        if out is not None:
            out.copy_(r)
            return out
        return r
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.long, device=logits.device)
    native().argmax_rows(out, logits)
    return out


def spec_verify(draft, target, seq_lens, out_tokens, accept, next_token) -> None:
    """Greedy accept/commit in place: seq_lens += accept + 1."""
    if not _cuda(draft):
        o, a, n, s = ref.spec_verify(draft, target, seq_lens)
        out_tokens.copy_(o)
        accept.copy_(a)
        next_token.copy_(n)
        seq_lens.copy_(s)
        return
    native().spec_verify(draft, target, seq_lens, out_tokens, accept, next_token)


# ----------------------------------------------------------------------------- GEMM
_GEMM_BACKEND = os.environ.get("SH_GEMM", "tcgen05")  # "cublas": library baseline for A/B runs


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ w.T for w [N, K].

    bf16 on a CUDA device runs the tcgen05 GEMM (K must be a multiple of 64);
    other dtypes (the fp32 toy model) and the CPU use the library matmul.
    """
    if x.is_cuda and x.dtype == torch.bfloat16 and _GEMM_BACKEND == "tcgen05":
        from .gemm import tcgen05_linear

        return tcgen05_linear(x, w, out)
    y = torch.matmul(x, w.t())
    if out is not None:
        out.copy_(y)
        return out
    return y
