"""DeepSeek-V3.2-style sparse-MLA MoE (config 3) and Kimi-K2 (config 4).

* MLA in its absorbed form: the cache holds the normalised latent c_kv
  (kv_lora) and the rotary key k_pe (rope) per token; queries are projected
  into the latent space with W_UK, attention runs over the latent rows, and
  W_UV maps the latent output back to per-head values.
* DSA lightning indexer (V3.2): per-token index keys are cached in fp8 pages
  (64 e4m3 keys of 128 bytes + 64 f32 key scales, 132 B per key); every query
  (quantised to e4m3 per head) scores its context with
  k_scale * sum_h relu(q_h . k) * w_h and attends only to the top-k positions.
* MoE: sigmoid group-limited router with score-correction bias, routed
  scaling, one shared expert; the first `first_dense_layers` layers are dense.
* Weights may be NVFP4 (ModelOpt layout: packed e2m1, e4m3 block-16 scales,
  fp32 global scale); dense NVFP4 linears dequantise into a scratch tile and
  run the tcgen05 GEMM.
"""
from __future__ import annotations

import math
from typing import List

import torch

from .. import ops
from ..parallel import comm, state
from .common import MLP, AttnMeta, Linear, RMSNorm, dtype_of, init_weight
from .moe import MoEBlock


class QLinear:
    """y = x W^T with W in bf16 or NVFP4.

    NVFP4 linears run the block-scaled W4A4 tcgen05 kernel on per-token NVFP4
    activations (static_g: the checkpoint's 1 / input_scale when it has one,
    else a per-token dynamic scale); SH_NVFP4_ACT=bf16 selects the W4A16
    kernel (packed weights decoded in shared memory).  `weight` (the dequantised matrix, for the MLA
    absorption of kv_b) decodes into one scratch tile per device shared by all
    NVFP4 layers (calls are ordered on the stream, so a captured graph replays
    them correctly).
    """

    _scratch: dict = {}

    def __init__(self, in_f: int, out_f: int, dtype, device, gen, fmt: str = "bf16", std: float = 0.02):
        w = init_weight((out_f, in_f), std, dtype, device, gen)
        self.fmt = fmt if in_f % (128 if fmt == "fp8" else 16) == 0 else "bf16"
        self.out_f, self.in_f, self.dtype = out_f, in_f, dtype
        if self.fmt == "fp8":  # MXFP8: e4m3 codes + ue8m0 scale per 32 (W8A8 block-scaled tcgen05 GEMM)
            self.codes, self.mx_scales = ops.mxfp8_quantize(w)
            self.w_sf = ops.mxfp8_scale_tiles(self.mx_scales) if self.codes.is_cuda else None
            self._w = None
        elif self.fmt == "nvfp4":
            self.packed, self.scales, self.gscale = ops.nvfp4_quantize(w)
            self.scales_k = ops.nvfp4_kmajor_scales(self.scales) if self.packed.is_cuda else None
            self.w_sf = ops.nvfp4_scale_tiles(self.scales) if self.packed.is_cuda else None
            self.static_g = 0.0
            self._w = None
            if self.packed.is_cuda:
                key = self.packed.device
                buf = QLinear._scratch.get(key)
                if buf is None or buf.numel() < out_f * in_f:
                    QLinear._scratch[key] = torch.empty(out_f * in_f, dtype=torch.bfloat16, device=key)
        else:
            self._w = w

    @property
    def weight(self) -> torch.Tensor:
        if self.fmt == "fp8":
            return ops.ref.mxfp8_dequantize(self.codes, self.mx_scales).to(self.dtype)
        if self.fmt != "nvfp4":
            return self._w
        if not self.packed.is_cuda:
            return ops.nvfp4_dequantize(self.packed, self.scales, self.gscale).to(self.dtype)
        out = QLinear._scratch[self.packed.device][: self.out_f * self.in_f].view(self.out_f, self.in_f)
        return ops.nvfp4_dequantize(self.packed, self.scales, self.gscale, out=out)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.fmt == "fp8" and x.dtype == torch.bfloat16:
            return ops.mxfp8_linear(x, self.codes, self.w_sf, self.mx_scales)
        if self.fmt == "nvfp4" and self.in_f % 64 == 0 and x.dtype == torch.bfloat16 and ops.nvfp4_act_mode() == "fp4":
            return ops.nvfp4_linear_w4a4(x, self.packed, self.w_sf, self.scales, self.gscale, self.static_g)
        if self.fmt == "nvfp4" and x.is_cuda and x.dtype == torch.bfloat16 and self.in_f % 64 == 0:
            return ops.nvfp4_linear(x, self.packed, self.scales, self.gscale, scales_k=self.scales_k)  # W4A16 kernel
        return ops.linear(x, self.weight)

    def refresh(self) -> None:
        """Rebuild the kernels' scale copies (k-block-major, block-scaled MMA tiles) after the packed
        weights changed."""
        if self.fmt == "nvfp4" and self.packed.is_cuda:
            self.scales_k = ops.nvfp4_kmajor_scales(self.scales)
            self.w_sf = ops.nvfp4_scale_tiles(self.scales)
        if self.fmt == "fp8" and self.codes.is_cuda:
            self.w_sf = ops.mxfp8_scale_tiles(self.mx_scales)

    def load(self, full: torch.Tensor) -> None:
        """Replace the weight by a full [out, in] matrix (re-quantised when the layer is NVFP4)."""
        if tuple(full.shape) != (self.out_f, self.in_f):
            raise ValueError(f"checkpoint matrix {tuple(full.shape)} != expected {(self.out_f, self.in_f)}")
        if self.fmt == "fp8":
            c, sc = ops.mxfp8_quantize(full.to(self.codes.device, torch.float32))
            self.codes.copy_(c)
            self.mx_scales.copy_(sc)
            self.refresh()
        elif self.fmt == "nvfp4":
            p, sc, g = ops.nvfp4_quantize(full.to(self.packed.device, self.dtype))
            self.packed.copy_(p)
            self.scales.copy_(sc)
            self.gscale.copy_(g)
            self.refresh()
        else:
            self._w.copy_(full.to(self._w.device, self._w.dtype))


class MLAttention:
    def __init__(self, cfg, dtype, device, gen, cos_sin, fmt: str):
        assert state.get().tp == 1, "MLA runs data-parallel (attention DP) with experts sharded by EP"
        self.cfg = cfg
        self.H = cfg.heads
        self.nope, self.rope, self.vd, self.lora = cfg.qk_nope, cfg.qk_rope, cfg.v_head, cfg.kv_lora
        self.kv_fp4 = cfg.kv_format == "nvfp4"  # NVFP4 latent cache (CUDA: packed rows; CPU: the same values)
        self.scale = ops.ref.yarn_softmax_mscale(cfg.rope_scaling) / math.sqrt(self.nope + self.rope)
        h = cfg.hidden
        self.q_a = QLinear(h, cfg.q_lora, dtype, device, gen, fmt) if cfg.q_lora else None
        self.q_a_norm = RMSNorm(cfg.q_lora, cfg.norm_eps, dtype, device) if cfg.q_lora else None
        self.q_b = QLinear(cfg.q_lora or h, self.H * (self.nope + self.rope), dtype, device, gen, fmt)
        self.kv_a = QLinear(h, self.lora + self.rope, dtype, device, gen, fmt)
        self.kv_a_norm = RMSNorm(self.lora, cfg.norm_eps, dtype, device)
        self.kv_b = QLinear(self.lora, self.H * (self.nope + self.vd), dtype, device, gen, fmt)
        self.o = QLinear(self.H * self.vd, h, dtype, device, gen, fmt)
        self.cos_sin = cos_sin
        self.dsa = cfg.dsa_topk > 0
        if self.dsa:
            self.ih, self.idim, self.itopk = cfg.dsa_heads, cfg.dsa_head_dim, cfg.dsa_topk
            self.idx_q = QLinear(cfg.q_lora or h, self.ih * self.idim, dtype, device, gen, fmt)
            self.idx_k = QLinear(h, self.idim, dtype, device, gen, fmt)
            self.idx_w = init_weight((self.ih, h), cfg.init_std, dtype, device, gen)

    def cache_width(self) -> int:
        return self.lora + self.rope

    def __call__(self, x: torch.Tensor, meta: AttnMeta, cache) -> torch.Tensor:
        latent, icache = cache[0], cache[1]
        tier = cache[2] if len(cache) > 2 else None  # host KV tier: `latent` is the host-resident cache
        T = x.shape[0]
        qa = self.q_a_norm(self.q_a(x)) if self.q_a is not None else x
        q = self.q_b(qa).view(T, self.H, self.nope + self.rope)
        ckv = self.kv_a(x)
        c = ops.rms_norm(ckv[:, : self.lora].contiguous(), self.kv_a_norm.weight, self.kv_a_norm.eps)
        kpe = ops.ref.apply_rope(ckv[:, self.lora:].reshape(T, 1, self.rope), meta.positions, self.cos_sin)[:, 0]
        q_pe = ops.ref.apply_rope(q[..., self.nope:], meta.positions, self.cos_sin)
        ops.mla_cache_write(latent, c, kpe.to(c.dtype), meta.slot_mapping, fp4=self.kv_fp4)
        wkv = self.kv_b.weight.view(self.H, self.nope + self.vd, self.lora)
        w_uk, w_uv = wkv[:, : self.nope], wkv[:, self.nope:]
        topk = None
        if self.dsa:
            qi = self.idx_q(qa).view(T, self.ih, self.idim)
            ki = self.idx_k(x)
            ops.dsa_cache_write(icache, ki.contiguous(), meta.slot_mapping)
            wt = ops.linear(x, self.idx_w).float() * (self.ih ** -0.5) * (self.idim ** -0.5)
            topk = ops.dsa_topk(qi, wt, icache, meta.block_tables, meta.seq_lens, meta.q_start, self.itopk)
        if x.is_cuda:
            # absorb W_UK into the queries (plain batched GEMMs), attention over the latent cache on this
            # framework's MLA kernel, then W_UV back to per-head values
            q_lat = torch.bmm(q[..., : self.nope].transpose(0, 1), w_uk).transpose(0, 1)
            qf = torch.cat([q_lat, q_pe.to(q_lat.dtype)], -1).contiguous()
            keys = meta.block_tables.shape[1] * latent.shape[1]
            lat, bt, seq, tk = latent, meta.block_tables, meta.seq_lens, topk
            if tier is not None and topk is not None and meta.window > 0:
                # decode: the selected keys' rows are resolved into this layer's hot rows on the device
                lat, bt, seq, tk = tier.resolve(topk.to(torch.int32).contiguous(), meta)
            o_lat = ops.mla_decode(qf, lat, bt, seq, meta.q_start, self.scale, self.lora, tk,
                                   ops.mla_splits(T, self.H, self.itopk if self.dsa else keys))
            o = torch.bmm(o_lat.transpose(0, 1), w_uv.transpose(1, 2)).transpose(0, 1)
            return self.o(o.reshape(T, self.H * self.vd).contiguous())
        q_lat = torch.einsum("thn,hnc->thc", q[..., : self.nope].float(), w_uk.float())
        o_lat = ops.ref.mla_attention(q_lat, q_pe, latent, meta.block_tables, meta.seq_lens, meta.q_start, self.scale,
                                      self.lora, topk)
        o = torch.einsum("thc,hvc->thv", o_lat, w_uv.float()).to(x.dtype)
        return self.o(o.reshape(T, self.H * self.vd))


class DeepseekLayer:
    def __init__(self, cfg, i: int, dtype, device, gen, cos_sin, fmt):
        self.input_norm = RMSNorm(cfg.hidden, cfg.norm_eps, dtype, device)
        self.attn = MLAttention(cfg, dtype, device, gen, cos_sin, fmt)
        self.post_norm = RMSNorm(cfg.hidden, cfg.norm_eps, dtype, device)
        self.ffn = MoEBlock(cfg, dtype, device, gen) if cfg.layer_is_moe(i) else MLP(cfg.hidden, cfg.ffn, dtype,
                                                                                   device, gen)

    def __call__(self, x, residual, meta, cache):
        h = self.attn(x, meta, cache)
        ops.fused_add_rms_norm(h, residual, self.post_norm.weight, self.post_norm.eps)
        return self.ffn(h)


class DeepseekModel:
    def __init__(self, cfg, device="cuda", seed: int = 0):
        self.cfg = cfg
        self.device = device
        self.dtype = dtype_of(cfg.dtype)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        self.gen = gen
        fmt = {"nvfp4": "nvfp4", "fp8_block": "fp8"}.get(cfg.weight_format, "bf16")
        self.cos_sin = ops.ref.rope_cos_sin(cfg.max_position, cfg.qk_rope, cfg.rope_theta, device=device,
                                              scaling=cfg.rope_scaling)
        self.embed = init_weight((cfg.vocab, cfg.hidden), cfg.init_std, self.dtype, device, gen)
        self.layers = [DeepseekLayer(cfg, i, self.dtype, device, gen, self.cos_sin, fmt) for i in range(cfg.layers)]
        self.norm = RMSNorm(cfg.hidden, cfg.norm_eps, self.dtype, device)
        self.lm_head = Linear(cfg.hidden, cfg.vocab, self.dtype, device, gen)
        self.vocab_offset = 0
        self.num_kv_layers = cfg.layers
        self.host_kv = None  # (hot rows, max positions, max decode tokens) with the host KV tier
        self.host_tier = None

    @property
    def kv_heads_local(self) -> int:
        return 1

    def kv_cache_shape(self, num_blocks: int, block_size: int):
        return (num_blocks, block_size, self.cfg.kv_lora + self.cfg.qk_rope)

    def _kv_fp4(self) -> bool:
        return self.cfg.kv_format == "nvfp4" and torch.device(self.device).type == "cuda"

    def _latent_row(self):
        """(row shape, dtype) of one latent cache row: NVFP4 bytes or kv_lora + rope values."""
        if self._kv_fp4():
            return (ops.mla_fp4_row_bytes(self.cfg.kv_lora, self.cfg.qk_rope),), torch.uint8
        return (self.cfg.kv_lora + self.cfg.qk_rope,), self.dtype

    def latent_block_bytes(self, block_size: int) -> int:
        shape, dt = self._latent_row()
        return block_size * shape[0] * torch.empty(0, dtype=dt).element_size()

    def kv_block_bytes(self, block_size: int) -> int:
        """Device bytes one KV block takes in one layer: the latent rows (NVFP4 or model dtype; on the host
        with the host KV tier) and, with the DSA indexer, its key page."""
        lat = 0 if self.host_kv is not None else self.latent_block_bytes(block_size)
        return lat + (ops.DSA_PAGE_BYTES if self.cfg.dsa_topk else 0)

    def enable_host_kv(self, hot_rows: int, max_positions: int, max_tokens: int) -> None:
        """Keep the target layers' latent caches in host memory with `hot_rows` device rows per request slot
        and layer (engine/host_tier.py); needs the DSA indexer (the hot rows hold each step's top-k keys)."""
        if not self.cfg.dsa_topk or torch.device(self.device).type != "cuda":
            raise ValueError("the host KV tier needs a DSA sparse-attention model on CUDA")
        self.host_kv = (hot_rows, max_positions, max_tokens)

    def allocate_caches(self, num_blocks: int, block_size: int, slots: int, window: int,
                        n_layers: int | None = None) -> List:
        if self.host_kv is not None and n_layers is None:  # the target's layers (the MTP layer stays on device)
            from ..engine.host_tier import HostKVTier

            hot_rows, max_pos, max_tok = self.host_kv
            shape, dt = self._latent_row()
            tier = HostKVTier(len(self.layers), num_blocks, block_size, shape, dt, slots, hot_rows, max_pos, max_tok,
                              self.cfg.dsa_topk, self.device)
            self.host_tier = tier
            return [(tier.cold[i], ops.dsa_cache_alloc(num_blocks, block_size, self.device), tier.layer(i))
                    for i in range(len(self.layers))]
        caches = []
        fp4 = self._kv_fp4()
        for _ in range(len(self.layers) if n_layers is None else n_layers):
            if fp4:  # NVFP4 latent rows (3.3x smaller than bf16 at kv_lora 512)
                lat = torch.zeros(num_blocks, block_size, ops.mla_fp4_row_bytes(self.cfg.kv_lora, self.cfg.qk_rope),
                                  dtype=torch.uint8, device=self.device)
            else:
                lat = torch.zeros(num_blocks, block_size, self.cfg.kv_lora + self.cfg.qk_rope, dtype=self.dtype,
                                  device=self.device)
            idx = ops.dsa_cache_alloc(num_blocks, block_size, self.device) if self.cfg.dsa_topk else None
            caches.append((lat, idx))
        return caches

    def forward(self, ids, meta: AttnMeta, caches, embeds=None):
        if self.host_tier is not None and meta.window == 0 and meta.state_slots is not None:
            self.host_tier.reset(meta.state_slots)  # prefill: these slots start new requests
        residual = ops.embedding(ids, self.embed) if embeds is None else embeds
        x = ops.rms_norm(residual, self.layers[0].input_norm.weight, self.cfg.norm_eps)
        for i, layer in enumerate(self.layers):
            m = layer(x, residual, meta, caches[i])
            nxt = self.layers[i + 1].input_norm if i + 1 < len(self.layers) else self.norm
            ops.fused_add_rms_norm(m, residual, nxt.weight, nxt.eps)
            x = m
        return x, residual

    def logits(self, hidden):
        return self.lm_head(hidden)

    def greedy(self, hidden, out=None):
        scr = getattr(self, "lm_screen", None)
        if scr is not None and scr.applies(hidden):  # NVFP4 screen + exact re-score (SUFFIX_NVFP4_LMHEAD)
            return comm.vocab_parallel_best(*scr.best(hidden), self.vocab_offset, out)
        return comm.vocab_parallel_argmax(self.logits(hidden), self.vocab_offset, out)


class DeepseekMtp:
    """One MTP layer (MLA + MoE) on [enorm(embed(token)), hnorm(feature)]; shares embedding and head."""

    def __init__(self, cfg, target: DeepseekModel, device="cuda"):
        self.cfg, self.target = cfg, target
        dt, gen = target.dtype, target.gen
        self.enorm = RMSNorm(cfg.hidden, cfg.norm_eps, dt, device)
        self.hnorm = RMSNorm(cfg.hidden, cfg.norm_eps, dt, device)
        self.eh_proj = init_weight((cfg.hidden, 2 * cfg.hidden), cfg.init_std, dt, device, gen)
        fmt = {"nvfp4": "nvfp4", "fp8_block": "fp8"}.get(cfg.weight_format, "bf16")
        self.layer = DeepseekLayer(cfg, cfg.layers, dt, device, gen, target.cos_sin, fmt)
        self.norm = RMSNorm(cfg.hidden, cfg.norm_eps, dt, device)

    def kv_block_bytes(self, block_size: int) -> int:
        # the MTP layer's cache is on the device even with the target's host KV tier
        t = self.target
        return t.latent_block_bytes(block_size) + (ops.DSA_PAGE_BYTES if self.cfg.dsa_topk else 0)

    def allocate_caches(self, num_blocks: int, block_size: int):
        return self.target.allocate_caches(num_blocks, block_size, 0, 0, n_layers=1)[0]

    def forward(self, tokens, feature, meta, cache):
        e = self.enorm(ops.embedding(tokens, self.target.embed))
        residual = ops.linear(torch.cat([e, self.hnorm(feature)], -1), self.eh_proj)
        x = ops.rms_norm(residual, self.layer.input_norm.weight, self.cfg.norm_eps)
        m = self.layer(x, residual, meta, cache)
        ops.fused_add_rms_norm(m, residual, self.norm.weight, self.norm.eps)
        return m, residual


def build(cfg, device, seed, with_draft):
    m = DeepseekModel(cfg, device, seed)
    return m, (DeepseekMtp(cfg, m, device) if with_draft else None)
