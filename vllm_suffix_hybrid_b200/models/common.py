"""Shared decoder building blocks (paged KV, tensor-parallel linears).

Weights are stored [out, in] like HF checkpoints; QKV and gate|up are fused
into one matrix each so one GEMM produces them.  Column-parallel layers keep
a contiguous slice of output rows per rank, row-parallel layers a slice of
input columns followed by an all-reduce (fused with the next residual-add +
RMSNorm when the fused comm runtime is active).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch

from .. import ops
from ..parallel import comm, state


def dtype_of(name: str) -> torch.dtype:
    return {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[name]


@dataclass
class AttnMeta:
    """Batch description for one forward over the paged cache."""

    positions: torch.Tensor  # [T] int64 absolute positions of the new tokens
    slot_mapping: torch.Tensor  # [T] int64 cache slots (-1: do not cache)
    block_tables: torch.Tensor  # [B, max_blocks] int32
    seq_lens: torch.Tensor  # [B] int64 length INCLUDING the new tokens
    q_start: torch.Tensor  # [B+1] int64 query start offsets
    tile_req: torch.Tensor  # [tiles] int32 (attention schedule)
    tile_row0: torch.Tensor  # [tiles] int32
    num_tokens: int = 0
    nsplit: int = 1  # KV splits per request (split-KV attention)
    max_rows: int = 64  # most valid rows in any 64-row query tile
    state_slots: Optional[torch.Tensor] = None  # [B] int64 recurrent-state slot per request
    pending: Optional[torch.Tensor] = None  # [slots] int32 accepted window records to replay
    window: int = 0  # verify-window length (0: prefill from an empty state)


def init_weight(shape, std: float, dtype, device, gen: Optional[torch.Generator]) -> torch.Tensor:
    w = torch.empty(shape, dtype=torch.float32 if device == "cpu" else dtype, device=device)
    w.normal_(0.0, std, generator=gen)
    return w.to(dtype)


class Linear:
    """y = x @ W^T with W [out, in]; `parallel` in {None, 'col', 'row'}.

    Random init draws the FULL matrix from the shared generator and keeps this
    rank's slice, so a TP=N model is the same function as the TP=1 model.
    `sections` splits a fused column-parallel output (QKV, gate|up) so each
    rank keeps its slice of every section.
    """

    def __init__(self, in_f: int, out_f: int, dtype, device, gen=None, std=0.02, parallel=None, sections=None):
        st = state.get()
        self.parallel = parallel if st.tp > 1 else None
        self.sections = sections
        self.full_shape = (out_f, in_f)
        self.weight = self.shard(init_weight((out_f, in_f), std, dtype, device, gen))
        self.out_f, self.in_f = self.weight.shape

    def shard(self, full: torch.Tensor) -> torch.Tensor:
        """This rank's slice of a full [out, in] matrix (identity without TP)."""
        st = state.get()
        out_f, in_f = full.shape
        if self.parallel == "col":
            secs = self.sections or [out_f]
            assert sum(secs) == out_f and all(s % st.tp == 0 for s in secs)
            parts, o = [], 0
            for s in secs:
                w = s // st.tp
                parts.append(full[o + st.tp_rank * w:o + (st.tp_rank + 1) * w])
                o += s
            return torch.cat(parts, 0).contiguous()
        if self.parallel == "row":
            assert in_f % st.tp == 0
            w = in_f // st.tp
            return full[:, st.tp_rank * w:(st.tp_rank + 1) * w].contiguous()
        return full.contiguous()

    def load(self, full: torch.Tensor) -> None:
        """Replace the weight by this rank's slice of a full [out, in] checkpoint matrix."""
        if tuple(full.shape) != tuple(self.full_shape):
            raise ValueError(f"checkpoint matrix {tuple(full.shape)} != expected {self.full_shape}")
        self.weight.copy_(self.shard(full.to(self.weight.device)).to(self.weight.dtype))

    push = True  # row-parallel: may push its rows to the owner ranks (finished by all_reduce_add_rms_norm)
    # Low-rank adapter (A [r, in_local], B [out_local, r], scale) of online draft tuning: y += scale * x A^T B^T,
    # added to this rank's (partial) output before any reduction; updated in place so captured graphs see it.
    lora = None

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None):
        if self.lora is not None:
            if out is None and self.parallel == "row":
                out = comm.partial_out(x.shape[0], self.out_f, x)
            y = ops.linear(x, self.weight, out)
            a, b, scale = self.lora
            y.add_(torch.matmul(torch.matmul(x, a.t()), b.t()), alpha=scale)
            return y
        if out is None and self.parallel == "row":
            if self.push and comm.can_push(x.shape[0], self.out_f, x):
                return comm.push_gemm(x, self.weight)  # reduce-scatter inside the GEMM epilogue
            out = comm.partial_out(x.shape[0], self.out_f, x)  # symmetric buffer under fused TP comm
        return ops.linear(x, self.weight, out)


class RMSNorm:
    def __init__(self, dim: int, eps: float, dtype, device):
        self.weight = torch.ones(dim, dtype=dtype, device=device)
        self.eps = eps

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rms_norm(x, self.weight, self.eps)


class Attention:
    """GQA attention with fused QKV, RoPE + cache write, paged attention, o_proj."""

    def __init__(self, cfg, dtype, device, gen, cos_sin: torch.Tensor):
        st = state.get()
        tp = st.tp
        assert cfg.heads % tp == 0 and cfg.kv_heads % tp == 0, "heads must divide by TP"
        self.hq = cfg.heads // tp
        self.hk = cfg.kv_heads // tp
        self.d = cfg.head_dim
        self.rot = int(cfg.head_dim * cfg.partial_rotary) // 2 * 2
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        h = cfg.hidden
        q_full, kv_full = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
        self.qkv = Linear(h, q_full + 2 * kv_full, dtype, device, gen, parallel="col",
                          sections=[q_full, kv_full, kv_full])
        self.o = Linear(cfg.heads * cfg.head_dim, h, dtype, device, gen, parallel="row")
        self.cos_sin = cos_sin

    def __call__(self, x: torch.Tensor, meta: AttnMeta, kv: tuple) -> torch.Tensor:
        qkv = self.qkv(x)
        k_cache, v_cache = kv
        ops.rope_kv_write(qkv, meta.positions, self.cos_sin, k_cache, v_cache, meta.slot_mapping, self.hq, self.hk,
                          self.d, self.rot)
        attn = torch.empty(x.shape[0], self.hq * self.d, dtype=x.dtype, device=x.device)
        ops.paged_attention(attn, qkv, k_cache, v_cache, meta.block_tables, meta.seq_lens, meta.q_start,
                            meta.tile_req, meta.tile_row0, self.hq, self.scale, meta.nsplit,
                            meta.max_rows)
        return self.o(attn)  # partial sum under TP (reduced by the caller)


class MLP:
    def __init__(self, hidden: int, ffn: int, dtype, device, gen):
        self.gate_up = Linear(hidden, 2 * ffn, dtype, device, gen, parallel="col", sections=[ffn, ffn])
        self.down = Linear(ffn, hidden, dtype, device, gen, parallel="row")

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        gu = self.gate_up(x)
        return self.down(ops.silu_mul(gu))


class DecoderLayer:
    def __init__(self, cfg, dtype, device, gen, cos_sin):
        self.input_norm = RMSNorm(cfg.hidden, cfg.norm_eps, dtype, device)
        self.attn = Attention(cfg, dtype, device, gen, cos_sin)
        self.post_norm = RMSNorm(cfg.hidden, cfg.norm_eps, dtype, device)
        self.mlp = MLP(cfg.hidden, cfg.ffn, dtype, device, gen)

    def __call__(self, x: torch.Tensor, residual: torch.Tensor, meta: AttnMeta, kv, first: bool):
        """x: the normalised input of this layer (residual holds the stream)."""
        h = self.attn(x, meta, kv)
        h = comm.all_reduce_add_rms_norm(h, residual, self.post_norm.weight, self.post_norm.eps,
                                         prefetch=self.mlp.gate_up.weight)
        m = self.mlp(h)
        return m  # partial; the next layer's input norm reduces + adds it


def sync_tp_weights(tensors: List[torch.Tensor]) -> None:
    """Replicated parameters must be identical on every TP rank."""
    import torch.distributed as dist

    st = state.get()
    if st.tp > 1:
        for t in tensors:
            dist.broadcast(t, src=0, group=st.group)
