"""Mixture-of-experts feed-forward block (Qwen3-Next, DeepSeek-V3.2, Kimi-K2).

Router -> top-k experts (softmax top-k, or sigmoid group-limited top-k with a
score-correction bias) -> expert-sorted grouped SwiGLU GEMMs on the tcgen05
tensor cores (device-side tile list, no host sync) -> weighted combine, plus
an optional shared expert (sigmoid-gated in Qwen3-Next).

Expert parallelism: with EP = N every rank holds E/N experts; tokens routed
to remote experts are handled by the all-to-all dispatch/combine of
:mod:`..parallel.ep` (the weights here are then this rank's local experts).
"""
from __future__ import annotations

import torch

from .. import ops
from ..parallel import comm, state
from .common import MLP, Linear, init_weight


def st_dp() -> int:
    return state.get().dp


class MoEBlock:
    def __init__(self, cfg, dtype, device, gen):
        st = state.get()
        self.cfg = cfg
        self.E = cfg.num_experts
        self.k = cfg.top_k
        self.F = cfg.expert_ffn
        self.H = cfg.hidden
        self.ep = st.ep
        self.E_local = self.E // max(self.ep, 1)
        self.gate = init_weight((self.E, cfg.hidden), cfg.init_std, dtype, device, gen)
        self.bias = (torch.zeros(self.E, dtype=torch.float32, device=device)
                     if cfg.router == "sigmoid_grouped" else None)
        # Experts stacked: w13 [E_local*2F, H] (gate rows then up rows), w2 [E_local*H, F].  Each
        # expert is drawn from its own seed, so the model is the same function for every EP size
        # and a rank only materialises its own experts.
        base = int(torch.randint(0, 2 ** 62, (1,), generator=gen, device=gen.device).item())
        e0 = st.ep_rank * self.E_local if self.ep > 1 else 0
        self.w13 = torch.empty(self.E_local * 2 * self.F, cfg.hidden, dtype=dtype, device=device)
        self.w2 = torch.empty(self.E_local * cfg.hidden, self.F, dtype=dtype, device=device)
        for j in range(self.E_local):
            g = torch.Generator(device=device)
            g.manual_seed(base + e0 + j)
            self.w13[j * 2 * self.F:(j + 1) * 2 * self.F] = init_weight((2 * self.F, cfg.hidden), cfg.init_std,
                                                                          dtype, device, g)
            self.w2[j * cfg.hidden:(j + 1) * cfg.hidden] = init_weight((cfg.hidden, self.F), cfg.init_std, dtype,
                                                                         device, g)
        # NVFP4 experts (weight_format nvfp4 on CUDA): packed codes + block scales + one global
        # scale per expert matrix; the grouped GEMMs run the block-scaled W4A4 tcgen05 kernel
        # (SH_NVFP4_ACT=bf16: the W4A16 kernel).
        self.fp4 = None
        if cfg.weight_format == "nvfp4" and torch.device(device).type == "cuda" and dtype == torch.bfloat16 \
                and cfg.hidden % 64 == 0 and self.F % 64 == 0:
            self.fp4 = (self._quant(self.w13, self.E_local, 2 * self.F), self._quant(self.w2, self.E_local, cfg.hidden))
            self.w13 = self.w2 = None  # the bf16 copies are dropped
        # MXFP8 experts (weight_format fp8_block on CUDA): e4m3 codes + ue8m0 scale per 32, W8A8 grouped GEMMs
        self.fp8 = None
        if self.fp4 is None and cfg.weight_format == "fp8_block" and torch.device(device).type == "cuda" \
                and dtype == torch.bfloat16 and cfg.hidden % 128 == 0 and self.F % 128 == 0:
            self.fp8 = tuple(self._quant8(w, r) for w, r in ((self.w13, 2 * self.F), (self.w2, cfg.hidden)))
            self.w13 = self.w2 = None
        self.shared = MLP(cfg.hidden, cfg.shared_ffn, dtype, device, gen) if cfg.shared_experts else None
        if self.shared is not None:
            self.shared.down.push = False  # reduced by a plain all-reduce below
        self.shared_gate = (init_weight((1, cfg.hidden), cfg.init_std, dtype, device, gen)
                            if cfg.shared_experts and cfg.arch == "qwen3_next" else None)

    @staticmethod
    def _quant(w: torch.Tensor, n_mat: int, rows: int):
        packed, scales, gs = [], [], []
        for e in range(n_mat):
            p, sc, g = ops.nvfp4_quantize(w[e * rows:(e + 1) * rows])
            packed.append(p)
            scales.append(sc)
            gs.append(g.reshape(1).float())
        sc = torch.cat(scales)
        return (torch.cat(packed), sc, torch.cat(gs), ops.nvfp4_kmajor_scales(sc), ops.nvfp4_scale_tiles(sc, rows))

    @staticmethod
    def _quant8(w: torch.Tensor, rows: int):
        codes, sc = ops.mxfp8_quantize(w)
        return codes, sc, ops.mxfp8_scale_tiles(sc, rows)

    def refresh(self) -> None:
        """Rebuild the kernels' scale copies (k-block-major for W4A16, block-scaled MMA tiles for W4A4)
        after the NVFP4 experts changed (checkpoint load)."""
        if self.fp4 is not None:
            rows = (2 * self.F, self.H)
            self.fp4 = tuple(q[:3] + (ops.nvfp4_kmajor_scales(q[1]), ops.nvfp4_scale_tiles(q[1], r))
                             for q, r in zip(self.fp4, rows))

    def router_logits(self, x: torch.Tensor) -> torch.Tensor:
        return ops.linear(x, self.gate).float() if not x.is_cuda else ops.linear(x, self.gate)

    def route_args(self) -> dict:
        """Selection parameters of ops.moe_route (besides logits and k)."""
        if self.cfg.router == "sigmoid_grouped":
            return dict(sigmoid_grouped=True, bias=self.bias, n_groups=self.cfg.n_groups,
                        topk_groups=self.cfg.topk_groups, renorm=True, scale=self.cfg.routed_scale)
        return dict(sigmoid_grouped=False, bias=None, n_groups=1, topk_groups=1, renorm=True, scale=1.0)

    def route(self, x: torch.Tensor):
        return ops.moe_route(self.router_logits(x), self.k, **self.route_args())

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """x: normalised input [T, H]; returns the (TP-partial-free) FFN output [T, H]."""
        if self.ep > 1 and st_dp() > 1:
            from ..parallel import ep

            if ep.a2a_enabled(x):  # the dispatch kernel runs the router top-k itself
                out = ep.dp_route_dispatch_combine(self, x, self.router_logits(x))
            else:
                ids, w = self.route(x)
                out = ep.dp_dispatch_combine(self, x, ids, w)
        elif self.ep > 1:
            from ..parallel import ep

            ids, w = self.route(x)
            out = ep.dispatch_combine(self, x, ids, w)
        else:
            ids, w = self.route(x)
            if self.fp4 is not None:
                out = ops.moe_experts_nvfp4(x, ids, w, self.fp4[0], self.fp4[1], self.E, self.F)
            elif self.fp8 is not None:
                out = ops.moe_experts_mxfp8(x, ids, w, self.fp8[0], self.fp8[1], self.E, self.F)
            else:
                out = ops.moe_experts(x, ids, w, self.w13, self.w2, self.E, self.F)
        if self.shared is not None:
            s = self.shared(x)
            if state.get().tp > 1:
                s = comm.all_reduce(s)
            if self.shared_gate is not None:
                g = torch.sigmoid(ops.linear(x, self.shared_gate).float())
                s = (s.float() * g).to(s.dtype)
            out = out + s
        return out
