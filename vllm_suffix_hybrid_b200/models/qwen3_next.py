"""Qwen3-Next-style hybrid MoE (config 2): Gated DeltaNet + gated attention.

Layers repeat `layer_pattern` (default "LLLA": three Gated DeltaNet layers,
then one gated full-attention layer); every layer's FFN is a MoE block
(softmax top-k routed experts + sigmoid-gated shared expert).  The draft
head is a one-layer MTP block with full attention.

Gated DeltaNet under speculative verify uses deferred commit: the verify
window's kernels write per-token records and leave the committed recurrent
and conv states untouched; the runner publishes `pending[slot] = accepted+1`
after verification and the next window first replays those records (see
csrc/kernels/gdn.cu).  A prefill run (mode 0) starts from zero state and
commits directly.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch

from .. import ops
from ..parallel import comm, state
from .common import AttnMeta, Linear, RMSNorm, dtype_of, init_weight
from .moe import MoEBlock


# Prefill runs through the chunked tensor-core kernel (SH_GDN_CHUNK=0: the recurrent kernel).
_CHUNKED = os.environ.get("SH_GDN_CHUNK", "1") != "0"


@dataclass
class GdnCache:
    state: torch.Tensor  # [slots, HV, V, K] fp32
    conv: torch.Tensor  # [slots, C, 3] fp32
    rec_x: torch.Tensor  # [slots, W, C]
    rec_k: torch.Tensor  # [slots, W, HV, K]
    rec_v: torch.Tensor  # [slots, W, HV, V]
    rec_g: torch.Tensor  # [slots, W, HV]
    rec_b: torch.Tensor  # [slots, W, HV]


class GdnLayer:
    def __init__(self, cfg, dtype, device, gen):
        assert state.get().tp == 1, "Gated DeltaNet layers run with TP=1 (expert parallelism shards the MoE)"
        self.H, self.HV, self.K = cfg.gdn_qk_heads, cfg.gdn_v_heads, cfg.gdn_head_dim
        self.C = 2 * self.H * self.K + self.HV * self.K
        self.eps = cfg.norm_eps
        self.in_qkvz = Linear(cfg.hidden, self.C + self.HV * self.K, dtype, device, gen)
        self.in_ba = Linear(cfg.hidden, 2 * self.HV, dtype, device, gen)
        self.conv_w = init_weight((self.C, cfg.gdn_conv), 0.5, torch.float32, device, gen)
        self.a_log = torch.log(torch.empty(self.HV, device=device).uniform_(1.0, 16.0, generator=gen))
        self.dt_bias = torch.full((self.HV,), 0.5, device=device)
        self.norm_w = torch.ones(self.K, dtype=dtype, device=device)
        self.out = Linear(self.HV * self.K, cfg.hidden, dtype, device, gen, parallel="row")

    def make_cache(self, slots: int, window: int, device) -> GdnCache:
        f = dict(dtype=torch.float32, device=device)
        return GdnCache(torch.zeros(slots, self.HV, self.K, self.K, **f), torch.zeros(slots, self.C, 3, **f),
                        torch.zeros(slots, window, self.C, **f), torch.zeros(slots, window, self.HV, self.K, **f),
                        torch.zeros(slots, window, self.HV, self.K, **f), torch.zeros(slots, window, self.HV, **f),
                        torch.zeros(slots, window, self.HV, **f))

    def __call__(self, x: torch.Tensor, meta: AttnMeta, cache: GdnCache) -> torch.Tensor:
        qkvz = self.in_qkvz(x)
        ba = self.in_ba(x)
        T = x.shape[0]
        y = torch.empty(T, self.C, dtype=x.dtype, device=x.device)
        mode = 1 if meta.window else 0
        W = cache.rec_x.shape[1]
        ops.gdn_conv(qkvz, self.conv_w, y, cache.conv, cache.rec_x, meta.pending, meta.state_slots, meta.q_start, W,
                     mode)
        o = torch.empty(T, self.HV * self.K, dtype=x.dtype, device=x.device)
        z = qkvz[:, self.C:]
        if mode == 0 and _CHUNKED and ops.gdn_chunk_ok(y, z, o, self.K):
            ops.gdn_chunk_prefill(y, z, ba, self.a_log, self.dt_bias, self.norm_w, cache.state, meta.state_slots,
                                  meta.q_start, o, self.H, self.HV, self.K, self.eps)
            return self.out(o)
        ops.gdn_recurrent(y, z, ba, self.a_log, self.dt_bias, self.norm_w, cache.state,
                          (cache.rec_k, cache.rec_v, cache.rec_g, cache.rec_b), meta.pending, meta.state_slots,
                          meta.q_start, o, self.H, self.HV, self.K, W, mode, self.eps)
        return self.out(o)


class GatedAttention:
    """Full attention with per-head q/k RMSNorm, partial rotary and a sigmoid output gate."""

    def __init__(self, cfg, dtype, device, gen, cos_sin):
        st = state.get()
        self.hq, self.hk, self.d = cfg.heads // st.tp, cfg.kv_heads // st.tp, cfg.head_dim
        self.rot = int(cfg.head_dim * cfg.partial_rotary) // 2 * 2
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        q, kv = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
        # Fused rows: q | k | v | gate so q,k,v stay contiguous for the cache/attention kernels.
        self.qkvg = Linear(cfg.hidden, 2 * q + 2 * kv, dtype, device, gen, parallel="col", sections=[q, kv, kv, q])
        self.q_norm = RMSNorm(cfg.head_dim, cfg.norm_eps, dtype, device)
        self.k_norm = RMSNorm(cfg.head_dim, cfg.norm_eps, dtype, device)
        self.o = Linear(q, cfg.hidden, dtype, device, gen, parallel="row")
        self.cos_sin = cos_sin

    def __call__(self, x: torch.Tensor, meta: AttnMeta, kv) -> torch.Tensor:
        T = x.shape[0]
        hq, hk, d = self.hq, self.hk, self.d
        qkvg = self.qkvg(x)
        ops.rms_norm_heads(qkvg[:, : hq * d].view(T, hq, d), self.q_norm.weight, self.q_norm.eps)
        ops.rms_norm_heads(qkvg[:, hq * d:(hq + hk) * d].view(T, hk, d), self.k_norm.weight, self.k_norm.eps)
        k_cache, v_cache = kv
        ops.rope_kv_write(qkvg, meta.positions, self.cos_sin, k_cache, v_cache, meta.slot_mapping, hq, hk, d,
                          self.rot)
        attn = torch.empty(T, hq * d, dtype=x.dtype, device=x.device)
        ops.paged_attention(attn, qkvg, k_cache, v_cache, meta.block_tables, meta.seq_lens, meta.q_start,
                            meta.tile_req, meta.tile_row0, hq, self.scale, meta.nsplit, meta.max_rows)
        gate = qkvg[:, (hq + 2 * hk) * d:(2 * hq + 2 * hk) * d]
        attn = (attn.float() * torch.sigmoid(gate.float())).to(x.dtype)
        return self.o(attn)


class HybridLayer:
    def __init__(self, cfg, kind: str, dtype, device, gen, cos_sin):
        self.kind = kind
        self.input_norm = RMSNorm(cfg.hidden, cfg.norm_eps, dtype, device)
        self.mixer = GdnLayer(cfg, dtype, device, gen) if kind == "L" else GatedAttention(cfg, dtype, device, gen,
                                                                                         cos_sin)
        self.post_norm = RMSNorm(cfg.hidden, cfg.norm_eps, dtype, device)
        self.moe = MoEBlock(cfg, dtype, device, gen)

    def __call__(self, x, residual, meta, cache):
        h = self.mixer(x, meta, cache)
        h = comm.all_reduce_add_rms_norm(h, residual, self.post_norm.weight, self.post_norm.eps)
        return self.moe(h)


class Qwen3NextModel:
    def __init__(self, cfg, device="cuda", seed: int = 0):
        self.cfg = cfg
        self.device = device
        self.dtype = dtype_of(cfg.dtype)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        self.gen = gen
        rot = int(cfg.head_dim * cfg.partial_rotary) // 2 * 2
        self.cos_sin = ops.ref.rope_cos_sin(cfg.max_position, rot, cfg.rope_theta, device=device, scaling=cfg.rope_scaling)
        self.embed = init_weight((cfg.vocab, cfg.hidden), cfg.init_std, self.dtype, device, gen)
        self.layers = [HybridLayer(cfg, cfg.layer_kind(i), self.dtype, device, gen, self.cos_sin)
                       for i in range(cfg.layers)]
        self.norm = RMSNorm(cfg.hidden, cfg.norm_eps, self.dtype, device)
        self.lm_head = Linear(cfg.hidden, cfg.vocab, self.dtype, device, gen, parallel="col")
        st = state.get()
        self.vocab_offset = st.tp_rank * self.lm_head.out_f if st.tp > 1 else 0
        self.has_recurrent_state = True

    @property
    def kv_heads_local(self) -> int:
        return self.cfg.kv_heads // state.get().tp

    @property
    def num_kv_layers(self) -> int:
        return sum(1 for l in self.layers if l.kind == "A")

    def kv_cache_shape(self, num_blocks: int, block_size: int):
        return (num_blocks, self.kv_heads_local, block_size, self.cfg.head_dim)

    def allocate_caches(self, num_blocks: int, block_size: int, slots: int, window: int) -> List:
        caches = []
        for l in self.layers:
            if l.kind == "A":
                shp = self.kv_cache_shape(num_blocks, block_size)
                caches.append((torch.zeros(shp, dtype=self.dtype, device=self.device),
                               torch.zeros(shp, dtype=self.dtype, device=self.device)))
            else:
                caches.append(l.mixer.make_cache(slots, window, self.device))
        return caches

    def forward(self, ids, meta: AttnMeta, caches, embeds=None):
        residual = ops.embedding(ids, self.embed) if embeds is None else embeds
        x = ops.rms_norm(residual, self.layers[0].input_norm.weight, self.cfg.norm_eps)
        for i, layer in enumerate(self.layers):
            m = layer(x, residual, meta, caches[i])
            nxt = self.layers[i + 1].input_norm if i + 1 < len(self.layers) else self.norm
            ops.fused_add_rms_norm(m, residual, nxt.weight, nxt.eps)  # MoE output is already complete
            x = m
        return x, residual

    def logits(self, hidden):
        return self.lm_head(hidden)

    def greedy(self, hidden, out=None):
        scr = getattr(self, "lm_screen", None)
        if scr is not None and scr.applies(hidden):  # NVFP4 screen + exact re-score (SUFFIX_NVFP4_LMHEAD)
            return comm.vocab_parallel_best(*scr.best(hidden), self.vocab_offset, out)
        return comm.vocab_parallel_argmax(self.logits(hidden), self.vocab_offset, out)


class MtpHead:
    """One-layer MTP draft (full gated attention + MoE) sharing embedding and LM head."""

    def __init__(self, cfg, target: Qwen3NextModel, device="cuda"):
        self.cfg = cfg
        self.target = target
        dt, gen = target.dtype, target.gen
        self.enorm = RMSNorm(cfg.hidden, cfg.norm_eps, dt, device)
        self.hnorm = RMSNorm(cfg.hidden, cfg.norm_eps, dt, device)
        self.fc = init_weight((cfg.hidden, 2 * cfg.hidden), cfg.init_std, dt, device, gen)
        self.layer = HybridLayer(cfg, "A", dt, device, gen, target.cos_sin)
        self.norm = RMSNorm(cfg.hidden, cfg.norm_eps, dt, device)

    def allocate_caches(self, num_blocks: int, block_size: int):
        shp = self.target.kv_cache_shape(num_blocks, block_size)
        return (torch.zeros(shp, dtype=self.target.dtype, device=self.target.device),
                torch.zeros(shp, dtype=self.target.dtype, device=self.target.device))

    def forward(self, tokens, feature, meta: AttnMeta, kv):
        e = self.enorm(ops.embedding(tokens, self.target.embed))
        f = self.hnorm(feature)
        residual = ops.linear(torch.cat([e, f], dim=-1), self.fc)
        x = ops.rms_norm(residual, self.layer.input_norm.weight, self.cfg.norm_eps)
        m = self.layer(x, residual, meta, kv)
        ops.fused_add_rms_norm(m, residual, self.norm.weight, self.norm.eps)
        return m, residual


def build(cfg, device, seed, with_draft):
    m = Qwen3NextModel(cfg, device, seed)
    return m, (MtpHead(cfg, m, device) if with_draft else None)
