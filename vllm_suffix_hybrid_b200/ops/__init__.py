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
    """KV splits per request (1..16).

    Splitting the keys lets short batches fill the SMs but costs a merge pass
    over fp32 partials (about a fifth of the attention time at decode sizes).
    With at least two waves of (tile, kv head) units the persistent kernel
    balances well enough unsplit, so splits are used only below that, sized
    for about four waves.  SH_ATTN_SPLITS forces a count.

    In batch-invariant mode (SH_BATCH_INVARIANT=1) the count depends on
    max_pages only, so a query row's merge order does not change with the
    number of other rows in the call.
    """
    if os.environ.get("SH_BATCH_INVARIANT", "0") == "1":
        return int(max(1, min(8, max_pages // 2)))
    forced = os.environ.get("SH_ATTN_SPLITS")
    if forced:
        return int(max(1, min(16, int(forced), max(1, max_pages // 2))))
    units = max(num_tiles * kv_heads, 1)
    if units >= 2 * sms:
        return 1
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
    native().embedding(out, ids.reshape(-1).contiguous(), table)
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


def spec_advance(out_tokens, accept, next_token, seq_new, cand, clen, native_drafts, win, seq, real,
                 hyb_min: int, real_batch: int) -> None:
    """Next verify window from this step's results and a lag-1 host candidate (async scheduling); in place
    into win [B, k+1], seq [B], real [B]; rows >= real_batch reset to the scratch window (see
    reference.spec_advance)."""
    if not _cuda(win):
        w, sq, rl = ref.spec_advance(out_tokens[: win.shape[0]], accept, next_token, seq_new, cand, clen,
                                     native_drafts, hyb_min)
        w[real_batch:] = 0
        sq[real_batch:] = 0
        rl[real_batch:] = 0
        win.copy_(w)
        seq.copy_(sq)
        real.copy_(rl)
        return
    nd = native_drafts.contiguous() if native_drafts is not None else None
    native().spec_advance(out_tokens, accept, next_token, seq_new, cand, clen, nd, win, seq, real, hyb_min,
                          real_batch)


# ----------------------------------------------------------------------------- GEMM
_GEMM_BACKEND = os.environ.get("SH_GEMM", "tcgen05")  # "cublas": library baseline for A/B runs


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ w.T for w [N, K].

    bf16 on a CUDA device runs the tcgen05 GEMM (K must be a multiple of 64);
    other dtypes (the fp32 toy model) and the CPU use the library matmul
    (fp32 on the CPU in batch-invariant mode: float64 accumulation).
    """
    if x.is_cuda and x.dtype == torch.bfloat16 and _GEMM_BACKEND == "tcgen05":
        from .gemm import tcgen05_linear

        return tcgen05_linear(x, w, out)
    if not x.is_cuda and x.dtype == torch.float32 and os.environ.get("SH_BATCH_INVARIANT", "0") == "1":
        # a row's result must not depend on the other rows of the call: float64 accumulation makes the
        # library's batch-size-dependent summation order invisible after rounding to fp32
        y = torch.matmul(x.double(), w.double().t()).to(x.dtype)
    else:
        y = torch.matmul(x, w.t())
    if out is not None:
        out.copy_(y)
        return out
    return y


# ----------------------------------------------------------------------------- Gated DeltaNet
def gdn_conv(x, w, y, state, rec_x, pending, slots, q_start, W: int, mode: int) -> None:
    """SiLU(causal depthwise conv) of x [T, >=C] into y [T, C]; mode 0 prefill (commits the taps),
    mode 1 verify window (replays `pending` records first, records this window's inputs)."""
    if x.is_cuda:
        native().gdn_conv(x, w, y, state, rec_x, pending, slots, q_start, W, mode)
        return
    C = w.shape[0]
    for b in range(slots.shape[0]):
        s = int(slots[b])
        t0, t1 = int(q_start[b]), int(q_start[b + 1])
        if mode == 0:
            st = torch.zeros(C, 3)
        else:
            st = state[s].clone()
            n = int(pending[s])
            if n:
                hist = torch.cat([st.t(), rec_x[s, :n]], 0)
                st = hist[-3:].t().contiguous()
                state[s] = st
        yb, new_st = ref.gdn_conv(x[t0:t1, :C], w, st)
        y[t0:t1] = yb.to(y.dtype)
        if mode == 0:
            state[s] = new_st
        else:
            rec_x[s, : t1 - t0] = x[t0:t1, :C].float()


def gdn_recurrent(qkv, z, ba, a_log, dt_bias, norm_w, state, rec, pending, slots, q_start, out, H, HV, K, W, mode,
                  eps) -> None:
    """Gated delta rule over each request's token run (see csrc/kernels/gdn.cu for the math)."""
    rec_k, rec_v, rec_g, rec_b = rec
    if qkv.is_cuda:
        native().gdn_recurrent(qkv, z, ba, a_log, dt_bias, norm_w, state, rec_k, rec_v, rec_g, rec_b, pending, slots,
                               q_start, out, H, HV, K, W, mode, eps)
        return
    rep = HV // H
    for b in range(slots.shape[0]):
        s = int(slots[b])
        t0, t1 = int(q_start[b]), int(q_start[b + 1])
        if mode == 0:
            S = torch.zeros(HV, K, K)
        else:
            S = state[s].clone()
            for r in range(int(pending[s])):
                ref.gdn_step(S, torch.zeros(HV, K), rec_k[s, r], rec_v[s, r], rec_g[s, r], rec_b[s, r])
            if int(pending[s]):
                state[s] = S
            S = S.clone()
        for t in range(t0, t1):
            row = qkv[t].float()
            q = ref.l2norm(row[: H * K].view(H, K)).repeat_interleave(rep, 0) * K ** -0.5
            k = ref.l2norm(row[H * K:2 * H * K].view(H, K)).repeat_interleave(rep, 0)
            v = row[2 * H * K:2 * H * K + HV * K].view(HV, K)
            g, beta = ref.gdn_gates(ba[t, HV:2 * HV], ba[t, :HV], a_log, dt_bias)
            o = ref.gdn_step(S, q, k, v, g, beta)
            if mode == 1:
                i = t - t0
                rec_k[s, i], rec_v[s, i], rec_g[s, i], rec_b[s, i] = k, v, g, beta
            out[t, : HV * K] = ref.gated_rms_norm(o, z[t, : HV * K].view(HV, K), norm_w, eps).reshape(-1).to(out.dtype)
        if mode == 0:
            state[s] = S


def gdn_chunk_prefill(qkv, z, ba, a_log, dt_bias, norm_w, state, slots, q_start, out, H, HV, K, eps,
                      err=None) -> None:
    """Prefill from zero state in 64-token chunks on the tensor cores (K == V == 128, rows 16-byte aligned):
    the same result as gdn_recurrent mode 0 up to bf16 rounding of the chunk products.  On the CPU it runs
    the recurrence."""
    if qkv.is_cuda:
        native().gdn_chunk_prefill(qkv, z, ba, a_log, dt_bias, norm_w, state, slots, q_start, out, H, HV, K, eps, err)
        return
    none = torch.zeros(0)
    gdn_recurrent(qkv, z, ba, a_log, dt_bias, norm_w, state, (none, none, none, none), None, slots, q_start, out, H,
                  HV, K, 0, 0, eps)


def gdn_chunk_ok(qkv, z, out, K: int) -> bool:
    """The chunked prefill applies: CUDA tensors, K == 128 and 16-byte aligned rows."""
    if not qkv.is_cuda or K != 128:
        return False
    return all(t.data_ptr() % 16 == 0 and (t.stride(0) * t.element_size()) % 16 == 0 for t in (qkv, z, out))


# ----------------------------------------------------------------------------- MoE
def moe_route(logits, k: int, sigmoid_grouped: bool = False, bias=None, n_groups: int = 1, topk_groups: int = 1,
              renorm: bool = True, scale: float = 1.0):
    """(ids int32 [T, k], weights f32 [T, k]) of the chosen experts."""
    T, E = logits.shape
    if logits.is_cuda:
        ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
        w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
        native().moe_route(logits, bias, ids, w, k, sigmoid_grouped, n_groups, topk_groups, renorm, scale)
        return ids, w
    lf = logits.float()
    if not sigmoid_grouped:
        p = lf.softmax(-1)
        w, ids = p.topk(k, dim=-1)
    else:
        sc = torch.sigmoid(lf)
        sb = sc + (bias.float() if bias is not None else 0.0)
        if n_groups > 1:
            g = sb.view(T, n_groups, -1)
            gs = g.topk(min(2, g.shape[-1]), dim=-1).values.sum(-1)
            keep = gs.topk(topk_groups, dim=-1).indices
            mask = torch.ones(T, n_groups, dtype=torch.bool)
            mask.scatter_(1, keep, False)
            sb = sb.masked_fill(mask.repeat_interleave(E // n_groups, 1), float("-inf"))
        ids = sb.topk(k, dim=-1).indices
        w = sc.gather(1, ids)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return ids.int(), (w * scale).float()


def moe_experts(x, ids, weights, w13, w2, E: int, F: int, out=None, accumulate: bool = False, push=None):
    """sum_j weights[t, j] * FFN_{ids[t, j]}(x[t]) with SwiGLU experts.

    w13: stacked [E*2F, H] (gate rows then up rows per expert), w2: [E*H, F]."""
    T, H = x.shape
    k = ids.shape[1]
    if not x.is_cuda:
        res = torch.zeros(T, H, dtype=torch.float32)
        for e in ids.unique().tolist():
            if e < 0 or e >= E:  # routed to another rank's experts
                continue
            tok, slot = (ids == e).nonzero(as_tuple=True)
            xe = x[tok].float()
            gu = xe @ w13[e * 2 * F:(e + 1) * 2 * F].float().t()
            a = torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
            ye = a.to(x.dtype).float() @ w2[e * H:(e + 1) * H].float().t()
            res.index_add_(0, tok, ye.to(x.dtype).float() * weights[tok, slot][:, None].float())
        if out is None:
            return res.to(x.dtype)
        if accumulate:
            out.copy_((out.float() + res).to(out.dtype))
        else:
            out.copy_(res.to(out.dtype))
        return out
    dev = x.device
    pairs = T * k
    bn = 64 if pairs <= E * 64 else 128
    max_groups = E + pairs // bn + 1
    C = native()
    rank = torch.empty(pairs, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    sorted_pos = torch.empty(pairs, dtype=torch.int32, device=dev)
    sorted_token = torch.zeros(pairs, dtype=torch.int32, device=dev)
    groups = torch.empty(max_groups, 4, dtype=torch.int32, device=dev)
    ngroups = torch.empty(1, dtype=torch.int32, device=dev)
    C.moe_align(ids, rank, offsets, sorted_pos, sorted_token, groups, ngroups, E, bn, 2 * F)
    xs = torch.empty(pairs, H, dtype=x.dtype, device=dev)
    C.moe_gather(xs, x, sorted_token, offsets[E:])
    gu = torch.empty(pairs, 2 * F, dtype=x.dtype, device=dev)
    C.gemm_grouped(gu, xs, w13, 2 * F, groups, ngroups, bn)
    a = silu_mul(gu)
    groups2 = groups.clone()
    groups2[:, 2] = groups[:, 3] * H  # down-projection weight row offsets
    ys = torch.empty(pairs, H, dtype=x.dtype, device=dev)
    C.gemm_grouped(ys, a, w2, H, groups2, ngroups, bn)
    if push is not None:  # the caller's combine takes the per-pair rows (expert-parallel combine push)
        push(ys, sorted_pos)
        return None
    if out is None:
        out = torch.empty(T, H, dtype=x.dtype, device=dev)
        accumulate = False
    C.moe_combine(out, ys, sorted_pos, weights, accumulate)
    return out


def rms_norm_heads(x3: torch.Tensor, w: torch.Tensor, eps: float) -> None:
    """In-place RMSNorm over the last dim of a [T, heads, D] strided view (q/k norms)."""
    if not x3.is_cuda:
        x3.copy_(ref.rms_norm(x3, w, eps))
        return
    T, nh, d = x3.shape
    tmp = x3.reshape(T * nh, d) if x3.is_contiguous() else x3.contiguous().view(T * nh, d)
    res = rms_norm(tmp, w, eps)
    x3.copy_(res.view(T, nh, d))


# ----------------------------------------------------------------------------- NVFP4
def nvfp4_quantize(w: torch.Tensor, global_scale: torch.Tensor | None = None):
    """bf16 [N, K] -> (packed uint8 [N, K/2], e4m3 scales [N, K/16], fp32 global [1])."""
    if global_scale is None:
        global_scale = ref.nvfp4_global_scale(w).to(w.device)
    if not w.is_cuda:
        p, s = ref.nvfp4_quantize(w, global_scale)
        return p, s, global_scale
    N, K = w.shape
    packed = torch.empty(N, K // 2, dtype=torch.uint8, device=w.device)
    scales = torch.empty(N, K // 16, dtype=torch.float8_e4m3fn, device=w.device)
    native().nvfp4_quant(packed, scales.view(torch.uint8), w.contiguous(), global_scale.float())
    return packed, scales, global_scale


def nvfp4_dequantize(packed, scales, global_scale, out: torch.Tensor | None = None) -> torch.Tensor:
    if not packed.is_cuda:
        r = ref.nvfp4_dequantize(packed, scales, global_scale)
        if out is not None:
            out.copy_(r)
            return out
        return r
    N, K = packed.shape[0], packed.shape[1] * 2
    if out is None:
        out = torch.empty(N, K, dtype=torch.bfloat16, device=packed.device)
    native().nvfp4_dequant(out, packed, scales.view(torch.uint8), global_scale.float())
    return out


# ----------------------------------------------------------------------------- MLA / DSA
_MLA_WS = {}


def mla_cache_write(latent: torch.Tensor, c: torch.Tensor, kpe: torch.Tensor, slots: torch.Tensor,
                    fp4: bool = False) -> None:
    """latent[slot] = [c | kpe] for every token with slot >= 0 (paged [blocks, 64, C] cache).  A uint8 cache
    holds NVFP4 latent rows (mla_fp4_row_bytes); on CPU, fp4=True stores the values such a cache returns."""
    if not latent.is_cuda:
        bs = latent.shape[1]
        ok = slots >= 0
        s = slots[ok]
        cc = ref.mla_fp4_qdq(c).to(c.dtype) if fp4 else c
        kk = ref.e4m3_qdq(kpe).to(c.dtype) if fp4 else kpe.to(c.dtype)
        latent[s // bs, s % bs] = torch.cat([cc, kk], -1)[ok].to(latent.dtype)
        return
    native().mla_cache_write(latent, c, kpe, slots)


def mla_fp4_row_bytes(kv_lora: int, rope: int) -> int:
    """Bytes of one NVFP4 latent cache row: kv_lora e2m1 values, the rope values in e4m3, kv_lora / 16 e4m3
    block scales, padded to 16 bytes (352 at kv_lora 512, rope 64; `reference.mla_fp4_pack` writes it)."""
    return (kv_lora // 2 + rope + kv_lora // 16 + 15) // 16 * 16


def mla_decode(q: torch.Tensor, latent: torch.Tensor, block_tables, seq_lens, q_start, scale: float, kv_lora: int,
               topk: torch.Tensor | None = None, nsplit: int = 1, stamps: torch.Tensor | None = None) -> torch.Tensor:
    """Absorbed MLA over the latent cache: q [T, H, C] -> o_lat [T, H, kv_lora] (bf16 on CUDA)."""
    if not q.is_cuda:
        return ref.mla_attention(q[..., :kv_lora], q[..., kv_lora:], latent, block_tables, seq_lens, q_start, scale,
                                 kv_lora, topk)
    T, H, C = q.shape
    out = torch.empty(T, H, kv_lora, dtype=torch.bfloat16, device=q.device)
    part_o = part_ml = None
    if nsplit > 1:
        idx = q.device.index if q.device.index is not None else torch.cuda.current_device()
        need_o, need_ml = T * H * nsplit * kv_lora, T * H * nsplit * 2
        ws = _MLA_WS.get(idx)
        if ws is None or ws[0].numel() < need_o or ws[1].numel() < need_ml:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("MLA split workspace must be sized before CUDA-graph capture")
            ws = (torch.empty(max(need_o, 1 << 16), dtype=torch.float32, device=q.device),
                  torch.empty(max(need_ml, 1 << 12), dtype=torch.float32, device=q.device))
            _MLA_WS[idx] = ws
        part_o, part_ml = ws
    err = torch.zeros(1, dtype=torch.int32, device=q.device)
    native().mla_decode(out, q.contiguous(), latent, block_tables, seq_lens, q_start,
                        None if topk is None else topk.to(torch.int32).contiguous(), nsplit, part_o, part_ml, scale,
                        err, 1 if os.environ.get("SH_MLA_TC", "1") == "0" else 0, stamps)
    return out


def mla_splits(num_tokens: int, heads: int, max_keys: int, sms: int = 148) -> int:
    if os.environ.get("SH_BATCH_INVARIANT", "0") == "1":
        return int(max(1, min(8, max_keys // 256)))
    units = max(num_tokens * -(-heads // 64), 1)
    return int(max(1, min(16, -(-sms // units), max(1, max_keys // 64))))


DSA_PAGE_KEYS = 64
DSA_DIM = 128
DSA_PAGE_BYTES = DSA_PAGE_KEYS * (DSA_DIM + 4)  # 64 e4m3 keys of 128 B, then 64 f32 key scales
_SMS = {}


def _num_sms(device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SMS[idx]


def dsa_cache_alloc(num_blocks: int, block_size: int, device) -> torch.Tensor:
    """Indexer key cache: one 8448-byte page (64 e4m3 keys + 64 f32 scales, 132 B per key) per block."""
    if block_size != DSA_PAGE_KEYS:
        raise ValueError(f"the indexer key cache needs {DSA_PAGE_KEYS}-token blocks, got {block_size}")
    return torch.zeros(num_blocks, DSA_PAGE_BYTES, dtype=torch.uint8, device=device)


def dsa_cache_write(cache: torch.Tensor, k: torch.Tensor, slots: torch.Tensor) -> None:
    """cache page slot // 64, row slot % 64 <- e4m3(k / s) with s = amax|k| / 448 stored as the key's scale."""
    if not cache.is_cuda:
        ref.dsa_cache_write(cache, k, slots)
        return
    native().dsa_cache_write(cache, k, slots)


def _dsa_ws(device, T: int, IH: int, max_keys: int):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = ("dsa", idx)
    ws = _MLA_WS.get(key)
    if ws is None or ws["q8"].shape[0] < T or ws["q8"].shape[1] != IH or ws["logits"].shape[1] < max_keys:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("indexer scratch must be sized before CUDA-graph capture")
        rows = max(T, 64)
        cols = -(-max(max_keys, 64) // 4) * 4
        ws = {"q8": torch.empty(rows, IH, DSA_DIM, dtype=torch.uint8, device=device),
              "wq": torch.empty(rows, IH, dtype=torch.float32, device=device),
              "logits": torch.empty(rows, cols, dtype=torch.float32, device=device),
              "err": torch.zeros(1, dtype=torch.int32, device=device)}
        _MLA_WS[key] = ws
    return ws


def dsa_topk(qi: torch.Tensor, w: torch.Tensor, kcache: torch.Tensor, block_tables, seq_lens, q_start,
             k: int, score_only: bool = False):
    """Lightning-indexer top-k positions per query token ([T, k] int32 ascending, -1 padded).

    qi [T, IH, 128] queries (quantised to e4m3 per (token, head) row here), w [T, IH] head weights, kcache
    the fp8 page cache of dsa_cache_alloc.  score_only returns the logits rows instead ([T, >= max_keys]
    fp32 scratch, row t valid on [0, pos_t]; a view of a reused buffer)."""
    if not qi.is_cuda:
        return ref.dsa_topk(qi, w, kcache, block_tables, seq_lens, q_start, k)
    T, IH = qi.shape[0], qi.shape[1]
    max_keys = block_tables.shape[1] * DSA_PAGE_KEYS
    ws = _dsa_ws(qi.device, T, IH, max_keys)
    q8, wq, logits = ws["q8"][:T], ws["wq"][:T], ws["logits"][:T]
    native().dsa_quant_q(q8, wq, qi.contiguous(), w.float().contiguous())
    out = logits if score_only else torch.empty(T, k, dtype=torch.int32, device=qi.device)
    native().dsa_index(out, logits, q8, wq, kcache, block_tables, seq_lens, q_start, _num_sms(qi.device), ws["err"],
                       score_only)
    return out


def nvfp4_kmajor_scales(scales: torch.Tensor) -> torch.Tensor:
    """ModelOpt block scales [N, K/16] -> the kernels' k-block-major layout [K/64, N_pad, 4] (N_pad: next
    multiple of 128), so one 64-wide k-block's scales of a 128-row tile are one contiguous 512-byte copy."""
    N, kb16 = scales.shape
    n_pad = -(-N // 128) * 128
    s8 = scales.view(torch.uint8).view(N, kb16 // 4, 4).permute(1, 0, 2)
    out = torch.zeros(kb16 // 4, n_pad, 4, dtype=torch.uint8, device=scales.device)
    out[:, :N] = s8
    return out


def nvfp4_linear(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, global_scale: torch.Tensor,
                 out: torch.Tensor | None = None, scales_k: torch.Tensor | None = None) -> torch.Tensor:
    """y = x W^T with W in NVFP4 (tcgen05 W4A16 kernel on CUDA; dequantised reference on CPU).

    The kernel reads the block scales in the k-block-major layout (`nvfp4_kmajor_scales`); layers keep
    that copy with their weights and pass it as scales_k (computed here otherwise)."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    N = packed.shape[0]
    if not x.is_cuda:
        w = ref.nvfp4_dequantize(packed, scales, global_scale).to(x.dtype)
        y = x2 @ w.t()
        return y.view(*lead, N)
    if x2.stride(-1) != 1 or (x2.stride(0) * 2) % 16 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    M = x2.shape[0]
    y = out.view(M, N) if out is not None else torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    if M:
        from .gemm import batch_invariant

        bn = 64 if M <= 64 else (128 if M <= 128 else 256)
        # split-K while the (weight tile x token tile) grid covers under half the SMs; in batch-invariant
        # mode the split count (which sets the fp32 summation order) is the one-token-tile choice for every M
        tiles = -(-N // 128) * (1 if batch_invariant() else -(-M // bn))
        kb = x2.shape[1] // 64
        splits = 1
        while tiles * splits * 2 <= 148 and kb // (splits * 2) >= 4 and splits < 16:
            splits *= 2
        from .gemm import workspace

        ws = workspace(x.device, splits * M * N) if splits > 1 else None
        sk = scales_k if scales_k is not None else nvfp4_kmajor_scales(scales)
        native().gemm_nvfp4(y, x2, packed, sk, global_scale.float().reshape(-1), bn, splits=splits, ws=ws)
    return y.view(*lead, N)


def nvfp4_act_mode() -> str:
    """How NVFP4 linears treat activations: "fp4" (default) quantises them to NVFP4 per token and runs
    the block-scaled W4A4 tensor-core GEMM (the serving math of ModelOpt NVFP4 checkpoints); "bf16"
    keeps bf16 activations (W4A16 kernel, weights decoded in shared memory).  SH_NVFP4_ACT selects."""
    return "bf16" if os.environ.get("SH_NVFP4_ACT", "fp4") == "bf16" else "fp4"


def nvfp4_scale_tiles(scales: torch.Tensor, rows_per_matrix: int | None = None) -> torch.Tensor:
    """ModelOpt block scales [R, K/16] -> the block-scaled MMA's scale tiles [R/rows_per_matrix * tiles,
    kc4, 512] (tiles = ceil(rows_per_matrix / 128) per matrix, kc4 = 4 * ceil(K / 256)): byte
    (r % 32) * 16 + (r / 32) * 4 + b % 4 of chunk b / 4 holds the scale of row r, 16-block b (zero padded)."""
    R, kb16 = scales.shape
    rp = rows_per_matrix or R
    nm = R // rp
    tp = -(-rp // 128)
    kc4 = -(-kb16 // 16) * 4
    buf = torch.zeros(nm, tp * 128, kc4 * 4, dtype=torch.uint8, device=scales.device)
    buf[:, :rp, :kb16] = scales.view(torch.uint8).reshape(nm, rp, kb16)
    return buf.view(nm * tp, 4, 32, kc4, 4).permute(0, 3, 2, 1, 4).contiguous().view(nm * tp, kc4, 512)


_FP4_ACT: dict = {}


def _fp4_act_buffers(dev, rows: int, K: int, tiles: int):
    """Per-device scratch of the activation quantiser (grown on demand, reused by every call)."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    kc4 = -(-K // 256) * 4
    b = _FP4_ACT.get(idx)
    if b is None or b[0].numel() < rows * K // 2 or b[1].numel() < tiles * kc4 * 512 or b[2].numel() < rows:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("NVFP4 activation scratch must be sized before CUDA-graph capture (run once eagerly)")
        old = (0, 0, 0) if b is None else (b[0].numel(), b[1].numel(), b[2].numel())
        b = (torch.empty(max(rows * K // 2, old[0], 1 << 20), dtype=torch.uint8, device=dev),
             torch.empty(max(tiles * kc4 * 512, old[1], 1 << 18), dtype=torch.uint8, device=dev),
             torch.empty(max(rows, old[2], 4096), dtype=torch.float32, device=dev))
        _FP4_ACT[idx] = b
    return (b[0][: rows * K // 2].view(rows, K // 2), b[1][: tiles * kc4 * 512].view(tiles, kc4, 512),
            b[2][:rows])


def nvfp4_quant_act(x: torch.Tensor, tile_rows: int, static_g: float = 0.0, groups=None, num_groups=None,
                    swiglu: bool = False):
    """(xq [R, K/2], x_sf scale tiles, a_scale [R]) of bf16 activations x [R, K] (see
    reference.nvfp4_quant_act); CUDA buffers are per-device scratch reused by the next call.  swiglu: x is a
    fused gate | up projection [R, 2K] and the quantised activation is silu_mul(x), fused into the kernel."""
    R, K = x.shape
    if swiglu:
        K //= 2
    tiles = groups.shape[0] if groups is not None else -(-R // tile_rows)
    xq, x_sf, a_scale = _fp4_act_buffers(x.device, R, K, tiles)
    native().nvfp4_quant_act(x, xq, x_sf, a_scale, tile_rows, float(static_g), groups, num_groups, swiglu)
    return xq, x_sf, a_scale


def nvfp4_gather_act(codes: torch.Tensor, scales: torch.Tensor, ascale: torch.Tensor, token: torch.Tensor,
                     groups: torch.Tensor, num_groups: torch.Tensor):
    """(xq, x_sf tiles, a_scale) of the grouped W4A4 operand built from rows already quantised to NVFP4
    (codes [R, K/2], e4m3 scales [R, K/16], a_scale [R]; reference.nvfp4_quant_act's layout): row r takes
    source row token[r].  Equal to nvfp4_quant_act of the gathered bf16 rows."""
    pairs, K = token.numel(), codes.shape[1] * 2
    xq, x_sf, a_scale = _fp4_act_buffers(codes.device, pairs, K, groups.shape[0])
    native().nvfp4_gather_act(codes, scales, ascale, token, groups, num_groups, xq, x_sf, a_scale)
    return xq, x_sf, a_scale


def nvfp4_linear_w4a4(x: torch.Tensor, packed: torch.Tensor, w_sf: torch.Tensor, scales: torch.Tensor,
                      global_scale: torch.Tensor, static_g: float = 0.0, out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x W^T with NVFP4 W and per-token NVFP4-quantised x (block-scaled tcgen05 MMA on CUDA; the fp32
    oracle of the same quantisation on CPU).  w_sf: `nvfp4_scale_tiles(scales)` kept with the weights."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    N = packed.shape[0]
    if not x.is_cuda:
        return ref.nvfp4_w4a4_linear(x2, packed, scales, global_scale, static_g).to(x.dtype).view(*lead, N)
    if x2.stride(-1) != 1 or (x2.stride(0) * 2) % 16 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    M, K = x2.shape
    y = out.view(M, N) if out is not None else torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    if M:
        bn = 64 if M <= 64 else 128
        xq, x_sf, a_scale = nvfp4_quant_act(x2, bn, static_g)
        splits, ws, cnt = _blockscaled_split(x.device, N, M, K, bn)
        native().gemm_fp4mma(y, xq, x_sf, a_scale, packed, w_sf, global_scale.float().reshape(-1), bn,
                             splits=splits, ws=ws, counters=cnt)
    return y.view(*lead, N)


def _blockscaled_split(dev, N: int, M: int, K: int, bn: int):
    """(splits, workspace, tickets) of a dense block-scaled GEMM (W4A4 / MXFP8) of reduction length K.

    K is split (in-kernel, the last split of a tile sums the fp32 partials in split order) while the tiles x
    splits cover at most half the SMs and every split keeps at least 1536 of K: below that the last split's
    reduction tail (about 5 us on B200) costs more than the shorter K loop saves (measured: a 7168-long K
    gains from 4 splits, a 2048-long K loses from 2).  Batch-invariant mode counts weight tiles only, so the
    split does not depend on M.  SH_FP4_SPLITK=0 turns splitting off."""
    from .gemm import batch_invariant, workspace

    tiles = -(-N // 128) * -(-M // bn)
    splits = 1
    if os.environ.get("SH_FP4_SPLITK", "1") != "0":
        t_split = -(-N // 128) if batch_invariant() else tiles
        while t_split * splits * 2 <= _num_sms(dev) and K // (splits * 2) >= 1536 and splits < 16:
            splits *= 2
    if splits == 1:
        return 1, None, None
    return splits, workspace(dev, splits * tiles * 128 * bn), split_tickets(dev, tiles)


_TICKETS: dict = {}


def split_tickets(dev, n: int) -> torch.Tensor:
    """Per-device zeroed int32 tickets of the in-kernel split-K reduction (each launch leaves them zero)."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    t = _TICKETS.get(idx)
    if t is None or t.numel() < n:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("split-K tickets must be sized before CUDA-graph capture (run once eagerly)")
        t = torch.zeros(max(n, 4096), dtype=torch.int32, device=dev)
        _TICKETS[idx] = t
    return t


def _moe_w4a4_cpu(x, ids, weights, w13q, w2q, E: int, F: int, out=None):
    """CPU oracle of the W4A4 expert path: per (token, expert) pair, quantise the input row, gate/up
    GEMM, SiLU * up in bf16, quantise again, down GEMM, weighted sum over the token's experts."""
    T, H = x.shape
    y = torch.zeros(T, H, dtype=torch.float32)
    for t in range(T):
        for j in range(ids.shape[1]):
            e = int(ids[t, j])
            if e < 0 or e >= E:
                continue
            r13 = slice(e * 2 * F, (e + 1) * 2 * F)
            gu = ref.nvfp4_w4a4_linear(x[t:t + 1], w13q[0][r13], w13q[1][r13], w13q[2][e:e + 1]).to(x.dtype)
            a = (torch.nn.functional.silu(gu[:, :F].float()) * gu[:, F:].float()).to(x.dtype)
            r2 = slice(e * H, (e + 1) * H)
            d = ref.nvfp4_w4a4_linear(a, w2q[0][r2], w2q[1][r2], w2q[2][e:e + 1]).to(x.dtype)
            y[t] += float(weights[t, j]) * d[0].float()
    y = y.to(x.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


# ----------------------------------------------------------------------------- MXFP8 (W8A8)
def _tile_layout(s8: torch.Tensor, rows_per_matrix: int, kc: int) -> torch.Tensor:
    """Per-row scale bytes [R, nblk] -> tensor-core scale tiles [matrices * tiles, kc, 512] (zero padded)."""
    R, nblk = s8.shape
    nm = R // rows_per_matrix
    tp = -(-rows_per_matrix // 128)
    buf = torch.zeros(nm, tp * 128, kc * 4, dtype=torch.uint8, device=s8.device)
    buf[:, :rows_per_matrix, :nblk] = s8.reshape(nm, rows_per_matrix, nblk)
    return buf.view(nm * tp, 4, 32, kc, 4).permute(0, 3, 2, 1, 4).contiguous().view(nm * tp, kc, 512)


def mxfp8_scale_tiles(scales: torch.Tensor, rows_per_matrix: int | None = None) -> torch.Tensor:
    """ue8m0 scales [R, K/32] -> scale tiles [R/rows_per_matrix * tiles, K/128, 512] of the MXFP8 GEMM."""
    R, nblk = scales.shape
    return _tile_layout(scales.view(torch.uint8), rows_per_matrix or R, -(-nblk // 4))


def mxfp8_quantize(w: torch.Tensor):
    """(e4m3 codes uint8 [R, K], ue8m0 scales [R, K/32]) of a matrix (load time; see reference)."""
    return ref.mxfp8_quantize(w)


def mxfp8_quant_act(x: torch.Tensor, tile_rows: int, groups=None, num_groups=None):
    R, K = x.shape
    tiles = groups.shape[0] if groups is not None else -(-R // tile_rows)
    dev = x.device
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    key = ("mx8", idx)
    b = _FP4_ACT.get(key)
    if b is None or b[0].numel() < R * K or b[1].numel() < tiles * (K // 128) * 512 or b[2].numel() < R:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("MXFP8 activation scratch must be sized before CUDA-graph capture (run once eagerly)")
        old = (0, 0, 0) if b is None else (b[0].numel(), b[1].numel(), b[2].numel())
        b = (torch.empty(max(R * K, old[0], 1 << 20), dtype=torch.uint8, device=dev),
             torch.empty(max(tiles * (K // 128) * 512, old[1], 1 << 18), dtype=torch.uint8, device=dev),
             torch.empty(max(R, old[2], 4096), dtype=torch.float32, device=dev))
        _FP4_ACT[key] = b
    xq, x_sf, a_sc = (b[0][: R * K].view(R, K), b[1][: tiles * (K // 128) * 512].view(tiles, K // 128, 512),
                      b[2][:R])
    native().mxfp8_quant_act(x, xq, x_sf, a_sc, tile_rows, groups, num_groups)
    return xq, x_sf, a_sc


_ONES: dict = {}


def _ones(dev, n: int) -> torch.Tensor:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    t = _ONES.get(idx)
    if t is None or t.numel() < n:
        t = torch.ones(max(n, 4096), dtype=torch.float32, device=dev)
        _ONES[idx] = t
    return t[:n]


def mxfp8_linear(x: torch.Tensor, codes: torch.Tensor, w_sf: torch.Tensor, scales: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x W^T with MXFP8 W (e4m3 + ue8m0 per 32) and per-32 MXFP8 x: block-scaled tcgen05 MMA
    (kind::mxf8f6f4) on CUDA, the fp32 oracle of the same quantisation on CPU."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    N = codes.shape[0]
    if not x.is_cuda:
        return ref.mxfp8_linear(x2, codes, scales).to(x.dtype).view(*lead, N)
    if x2.stride(-1) != 1 or (x2.stride(0) * 2) % 16 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    M = x2.shape[0]
    y = out.view(M, N) if out is not None else torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    if M:
        bn = 64 if M <= 64 else 128
        xq, x_sf, a_sc = mxfp8_quant_act(x2, bn)
        splits, ws, cnt = _blockscaled_split(x.device, N, M, x2.shape[1], bn)
        native().gemm_fp4mma(y, xq, x_sf, a_sc, codes, w_sf, _ones(x.device, 1), bn, splits=splits, ws=ws,
                             counters=cnt, fp8=True)
    return y.view(*lead, N)


def moe_experts_mxfp8(x, ids, weights, w13q, w2q, E: int, F: int, out=None, push=None):
    """MoE experts with MXFP8 weights: w13q = (codes [E*2F, H], scales [E*2F, H/32], scale tiles), w2q likewise
    for [E*H, F]; grouped block-scaled W8A8 GEMMs (CPU: fp32 oracle per pair)."""
    T, H = x.shape
    if not x.is_cuda:
        y = torch.zeros(T, H, dtype=torch.float32)
        for t in range(T):
            for j in range(ids.shape[1]):
                e = int(ids[t, j])
                if e < 0 or e >= E:
                    continue
                r13, r2 = slice(e * 2 * F, (e + 1) * 2 * F), slice(e * H, (e + 1) * H)
                gu = ref.mxfp8_linear(x[t:t + 1], w13q[0][r13], w13q[1][r13]).to(x.dtype)
                a = (torch.nn.functional.silu(gu[:, :F].float()) * gu[:, F:].float()).to(x.dtype)
                y[t] += float(weights[t, j]) * ref.mxfp8_linear(a, w2q[0][r2], w2q[1][r2])[0].to(x.dtype).float()
        y = y.to(x.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    k = ids.shape[1]
    dev = x.device
    pairs = T * k
    bn = 64 if pairs <= E * 64 else 128
    max_groups = E + pairs // bn + 1
    C = native()
    rank = torch.empty(pairs, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    sorted_pos = torch.empty(pairs, dtype=torch.int32, device=dev)
    sorted_token = torch.zeros(pairs, dtype=torch.int32, device=dev)
    groups = torch.empty(max_groups, 4, dtype=torch.int32, device=dev)
    ngroups = torch.empty(1, dtype=torch.int32, device=dev)
    C.moe_align(ids, rank, offsets, sorted_pos, sorted_token, groups, ngroups, E, bn, 2 * F)
    xs = torch.empty(pairs, H, dtype=x.dtype, device=dev)
    C.moe_gather(xs, x, sorted_token, offsets[E:])
    gu = torch.empty(pairs, 2 * F, dtype=x.dtype, device=dev)
    groups2 = groups.clone()
    groups2[:, 2] = groups[:, 3] * H
    ys = torch.empty(pairs, H, dtype=x.dtype, device=dev)
    t13 = w13q[2] if len(w13q) > 2 else mxfp8_scale_tiles(w13q[1], 2 * F)
    t2 = w2q[2] if len(w2q) > 2 else mxfp8_scale_tiles(w2q[1], H)
    ones = _ones(dev, E)
    xq, x_sf, a_sc = mxfp8_quant_act(xs, bn, groups, ngroups)
    C.gemm_fp4mma(gu, xq, x_sf, a_sc, w13q[0], t13, ones, bn, groups, ngroups, 2 * F, fp8=True)
    a = silu_mul(gu)
    xq, x_sf, a_sc = mxfp8_quant_act(a, bn, groups, ngroups)
    C.gemm_fp4mma(ys, xq, x_sf, a_sc, w2q[0], t2, ones, bn, groups2, ngroups, H, fp8=True)
    if push is not None:
        push(ys, sorted_pos)
        return None
    if out is None:
        out = torch.empty(T, H, dtype=x.dtype, device=dev)
    C.moe_combine(out, ys, sorted_pos, weights, False)
    return out


def moe_experts_nvfp4(x, ids, weights, w13q, w2q, E: int, F: int, out=None, prequant=None, push=None):
    """moe_experts with NVFP4 expert weights: w13q = (packed [E*2F, H/2], scales [E*2F, H/16], global [E],
    optional k-block-major scales, optional block-scaled MMA scale tiles), w2q likewise for [E*H, F].
    The grouped GEMMs run the block-scaled W4A4 tcgen05 kernel on per-token NVFP4 activations (or the
    W4A16 kernel with SH_NVFP4_ACT=bf16), each expert's rows scaled by its global scale.  On CPU the
    W4A4 mode quantises the activations like the kernel and multiplies dequantised values in fp32.
    prequant = (codes [T, H/2], scales [T, H/16], a_scale [T]): the rows arrive already quantised (the
    quantising expert-parallel dispatch); x is then unused (W4A4 on CUDA only)."""
    if prequant is not None:
        if not ids.is_cuda or nvfp4_act_mode() != "fp4":
            raise ValueError("pre-quantised expert input needs the CUDA W4A4 path")
        T, H = ids.shape[0], prequant[0].shape[1] * 2
    else:
        T, H = x.shape
    if prequant is None and not x.is_cuda and nvfp4_act_mode() == "fp4":
        return _moe_w4a4_cpu(x, ids, weights, w13q, w2q, E, F, out)
    if prequant is None and not x.is_cuda:
        w13 = torch.cat([ref.nvfp4_dequantize(w13q[0][e * 2 * F:(e + 1) * 2 * F], w13q[1][e * 2 * F:(e + 1) * 2 * F],
                                              w13q[2][e:e + 1]) for e in range(E)]).to(x.dtype)
        w2 = torch.cat([ref.nvfp4_dequantize(w2q[0][e * H:(e + 1) * H], w2q[1][e * H:(e + 1) * H], w2q[2][e:e + 1])
                        for e in range(E)]).to(x.dtype)
        return moe_experts(x, ids, weights, w13, w2, E, F, out=out)
    k = ids.shape[1]
    dev = ids.device
    pairs = T * k
    bn = 64 if pairs <= E * 64 else 128
    max_groups = E + pairs // bn + 1
    C = native()
    rank = torch.empty(pairs, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    sorted_pos = torch.empty(pairs, dtype=torch.int32, device=dev)
    sorted_token = torch.zeros(pairs, dtype=torch.int32, device=dev)
    groups = torch.empty(max_groups, 4, dtype=torch.int32, device=dev)
    ngroups = torch.empty(1, dtype=torch.int32, device=dev)
    C.moe_align(ids, rank, offsets, sorted_pos, sorted_token, groups, ngroups, E, bn, 2 * F)
    dt = torch.bfloat16
    if prequant is None:
        xs = torch.empty(pairs, H, dtype=dt, device=dev)
        C.moe_gather(xs, x, sorted_token, offsets[E:])
    gu = torch.empty(pairs, 2 * F, dtype=dt, device=dev)
    groups2 = groups.clone()
    groups2[:, 2] = groups[:, 3] * H
    ys = torch.empty(pairs, H, dtype=dt, device=dev)
    if nvfp4_act_mode() == "fp4":
        # W4A4: each group entry's activation rows are quantised into the entry's own scale tile
        t13 = w13q[4] if len(w13q) > 4 else nvfp4_scale_tiles(w13q[1], 2 * F)
        t2 = w2q[4] if len(w2q) > 4 else nvfp4_scale_tiles(w2q[1], H)
        if prequant is not None:
            xq, x_sf, a_sc = nvfp4_gather_act(prequant[0], prequant[1], prequant[2], sorted_token, groups, ngroups)
        else:
            xq, x_sf, a_sc = nvfp4_quant_act(xs, bn, 0.0, groups, ngroups)
        C.gemm_fp4mma(gu, xq, x_sf, a_sc, w13q[0], t13, w13q[2], bn, groups, ngroups, 2 * F)
        xq, x_sf, a_sc = nvfp4_quant_act(gu, bn, 0.0, groups, ngroups, swiglu=True)  # SwiGLU fused into the quantiser
        C.gemm_fp4mma(ys, xq, x_sf, a_sc, w2q[0], t2, w2q[2], bn, groups2, ngroups, H)
    else:
        sk13 = w13q[3] if len(w13q) > 3 and w13q[3] is not None else nvfp4_kmajor_scales(w13q[1])
        sk2 = w2q[3] if len(w2q) > 3 and w2q[3] is not None else nvfp4_kmajor_scales(w2q[1])
        C.gemm_nvfp4(gu, xs, w13q[0], sk13, w13q[2], bn, groups, ngroups, 2 * F)
        a = silu_mul(gu)
        C.gemm_nvfp4(ys, a, w2q[0], sk2, w2q[2], bn, groups2, ngroups, H)
    if push is not None:
        push(ys, sorted_pos)
        return None
    if out is None:
        out = torch.empty(T, H, dtype=dt, device=dev)
    C.moe_combine(out, ys, sorted_pos, weights, False)
    return out
