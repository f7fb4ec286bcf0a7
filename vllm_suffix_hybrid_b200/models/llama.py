"""Llama-family dense decoder (config 0 toy and config 1 Llama-3-8B shape).

Embedding and final norm are replicated; attention/MLP are tensor-parallel;
the LM head is vocab-parallel and greedy decoding reduces it to a global
argmax without gathering logits.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from .. import ops
from ..parallel import comm, state
from .common import AttnMeta, DecoderLayer, Linear, RMSNorm, dtype_of, init_weight


class LlamaModel:
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
        self.layers = [DecoderLayer(cfg, self.dtype, device, gen, self.cos_sin) for _ in range(cfg.layers)]
        self.norm = RMSNorm(cfg.hidden, cfg.norm_eps, self.dtype, device)
        st = state.get()
        self.lm_head = Linear(cfg.hidden, cfg.vocab, self.dtype, device, gen, parallel="col")
        self.vocab_offset = st.tp_rank * self.lm_head.out_f if st.tp > 1 else 0

    # -- shapes ---------------------------------------------------------------
    @property
    def kv_heads_local(self) -> int:
        return self.cfg.kv_heads // state.get().tp

    def kv_cache_shape(self, num_blocks: int, block_size: int) -> Tuple[int, ...]:
        return (num_blocks, self.kv_heads_local, block_size, self.cfg.head_dim)

    # -- forward --------------------------------------------------------------
    def forward(self, ids: torch.Tensor, meta: AttnMeta, kv_caches: List[tuple],
                embeds: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Returns (normed final hidden [T, H], pre-norm final hidden [T, H])."""
        residual = ops.embedding(ids, self.embed) if embeds is None else embeds
        x = ops.rms_norm(residual, self.layers[0].input_norm.weight, self.cfg.norm_eps)
        for i, layer in enumerate(self.layers):
            m = layer(x, residual, meta, kv_caches[i], i == 0)
            last = i + 1 == len(self.layers)
            nxt = self.norm if last else self.layers[i + 1].input_norm
            x = comm.all_reduce_add_rms_norm(m, residual, nxt.weight, nxt.eps, gather_residual=last,
                                             prefetch=None if last else self.layers[i + 1].attn.qkv.weight)
        return x, residual

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.lm_head(hidden)

    def greedy(self, hidden: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        scr = getattr(self, "lm_screen", None)
        if scr is not None and scr.applies(hidden):  # NVFP4 screen + exact re-score (SUFFIX_NVFP4_LMHEAD)
            return comm.vocab_parallel_best(*scr.best(hidden), self.vocab_offset, out)
        return comm.vocab_parallel_argmax(self.logits(hidden), self.vocab_offset, out)


class DraftHead:
    """One-layer draft head sharing the target's embedding and LM head.

    style 'eagle': x = fc([embed(token), feature]); 'mtp': the embedding and
    the feature are RMS-normalised before the projection.  The feature is the
    target's pre-norm final hidden state at the previous position (first
    step) or the head's own output (later steps).
    """

    def __init__(self, cfg, target: LlamaModel, device="cuda", style: str = "eagle"):
        self.cfg = cfg
        self.target = target
        self.style = style
        dt = target.dtype
        gen = target.gen
        self.fc = init_weight((cfg.hidden, 2 * cfg.hidden), cfg.init_std, dt, device, gen)
        self.enorm = RMSNorm(cfg.hidden, cfg.norm_eps, dt, device)
        self.hnorm = RMSNorm(cfg.hidden, cfg.norm_eps, dt, device)
        self.layer = DecoderLayer(cfg, dt, device, gen, target.cos_sin)
        self.norm = RMSNorm(cfg.hidden, cfg.norm_eps, dt, device)

    def forward(self, tokens: torch.Tensor, feature: torch.Tensor, meta: AttnMeta, kv: tuple):
        e = ops.embedding(tokens, self.target.embed)
        if self.style == "mtp":
            e = self.enorm(e)
            feature = self.hnorm(feature)
        residual = ops.linear(torch.cat([e, feature], dim=-1), self.fc)
        x = ops.rms_norm(residual, self.layer.input_norm.weight, self.cfg.norm_eps)
        m = self.layer(x, residual, meta, kv, True)
        x = comm.all_reduce_add_rms_norm(m, residual, self.norm.weight, self.norm.eps, gather_residual=True)
        return x, residual  # (normed, pre-norm feature for the next step)
