"""Plain PyTorch (fp32-accumulating) statements of every kernel's math.

These are the numerics oracles for the CUDA kernels and the execution path
of the CPU-only toy configuration.  They are written for clarity, not speed.
"""
from __future__ import annotations

import math
from typing import Optional

import torch


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * inv * w.float()).to(x.dtype)


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float) -> None:
    s = (x.float() + residual.float()).to(residual.dtype)
    residual.copy_(s)
    x.copy_(rms_norm(s, w, eps))


def rope_inv_freq(rot: int, theta: float, scaling: Optional[dict] = None):
    """(inverse frequencies [rot/2] float64, cos/sin attention factor) for plain, llama3 or YaRN RoPE.

    llama3: wavelengths above original_ctx / low_freq_factor are divided by
    `factor`, those below original_ctx / high_freq_factor kept, a linear blend
    in between.  YaRN (Peng et al. 2023, arXiv:2309.00071): per-dimension blend
    of interpolated (/factor) and extrapolated frequencies with a linear ramp
    between the correction dims of beta_fast and beta_slow rotations, and
    cos/sin scaled by 0.1 * mscale * ln(factor) + 1 (ratio of the mscale and
    mscale_all_dim terms when both are given).
    """
    inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.float64) / rot))
    kind = (scaling or {}).get("rope_type", (scaling or {}).get("type", "default"))
    if kind in (None, "default"):
        return inv, 1.0
    factor = float(scaling["factor"])
    if kind == "llama3":
        old = float(scaling["original_max_position_embeddings"])
        lo, hi = float(scaling["low_freq_factor"]), float(scaling["high_freq_factor"])
        wl = 2 * math.pi / inv
        smooth = ((old / wl) - lo) / (hi - lo)
        out = torch.where(wl > old / lo, inv / factor, inv)
        mid = (wl <= old / lo) & (wl >= old / hi)
        return torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, out), 1.0
    if kind == "yarn":
        old = float(scaling["original_max_position_embeddings"])
        beta_fast = float(scaling.get("beta_fast") or 32)
        beta_slow = float(scaling.get("beta_slow") or 1)

        def corr_dim(rotations):
            return (rot * math.log(old / (rotations * 2 * math.pi))) / (2 * math.log(theta))

        lo, hi = math.floor(corr_dim(beta_fast)), math.ceil(corr_dim(beta_slow))
        if scaling.get("truncate", True) is False:
            lo, hi = corr_dim(beta_fast), corr_dim(beta_slow)
        lo, hi = max(lo, 0), min(hi, rot - 1)
        if lo == hi:
            hi += 0.001
        ramp = ((torch.arange(rot // 2, dtype=torch.float64) - lo) / (hi - lo)).clamp(0, 1)
        extrap = 1 - ramp
        inv = (inv / factor) * (1 - extrap) + inv * extrap

        def mscale(s, m=1.0):
            return 1.0 if s <= 1 else 0.1 * m * math.log(s) + 1.0

        att = scaling.get("attention_factor")
        if att is None:
            m, mad = scaling.get("mscale"), scaling.get("mscale_all_dim")
            att = mscale(factor, m) / mscale(factor, mad) if (m and mad) else mscale(factor)
        return inv, float(att)
    raise ValueError(f"unsupported rope scaling {kind!r}")


def rope_cos_sin(max_pos: int, rot: int, theta: float, device=None, scaling: Optional[dict] = None) -> torch.Tensor:
    """[max_pos, rot] float32: cos in the first rot/2 columns, sin in the rest (scaled RoPE supported)."""
    inv, att = rope_inv_freq(rot, theta, scaling)
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return (torch.cat([f.cos(), f.sin()], dim=-1) * att).float().to(device)


def yarn_softmax_mscale(scaling: Optional[dict]) -> float:
    """DeepSeek-style extra softmax scale factor (mscale_all_dim term squared) under YaRN."""
    if not scaling or scaling.get("rope_type", scaling.get("type")) != "yarn":
        return 1.0
    mad = scaling.get("mscale_all_dim")
    factor = float(scaling["factor"])
    if not mad or factor <= 1:
        return 1.0
    m = 0.1 * float(mad) * math.log(factor) + 1.0
    return m * m


def apply_rope(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """x: [T, H, D]; rotate-half rotary on the first `rot` dims."""
    rot = cos_sin.shape[1]
    half = rot // 2
    cs = cos_sin[positions]
    c, s = cs[:, None, :half], cs[:, None, half:]
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:rot]
    out = xf.clone()
    out[..., :half] = x1 * c - x2 * s
    out[..., half:rot] = x2 * c + x1 * s
    return out.to(x.dtype)


def rope_kv_write(qkv, positions, cos_sin, k_cache, v_cache, slot_mapping, hq, hk, d, rot) -> None:
    t = qkv.shape[0]
    q = qkv[:, : hq * d].view(t, hq, d)
    k = qkv[:, hq * d:(hq + hk) * d].view(t, hk, d)
    v = qkv[:, (hq + hk) * d:(hq + 2 * hk) * d].view(t, hk, d)
    q.copy_(apply_rope(q, positions, cos_sin))
    k.copy_(apply_rope(k, positions, cos_sin))
    bs = k_cache.shape[2]
    ok = slot_mapping >= 0
    slots = slot_mapping[ok]
    blk, off = slots // bs, slots % bs
    k_cache[blk, :, off, :] = k[ok]
    v_cache[blk, :, off, :] = v[ok]


def paged_attention(q, k_cache, v_cache, block_tables, seq_lens, q_start, hq, scale) -> torch.Tensor:
    """q: [T, hq, D]; caches [blocks, hk, bs, D]; returns [T, hq, D]."""
    hk, bs, d = k_cache.shape[1], k_cache.shape[2], k_cache.shape[3]
    g = hq // hk
    out = torch.zeros_like(q)
    for b in range(seq_lens.shape[0]):
        s0, s1 = int(q_start[b]), int(q_start[b + 1])
        ql, sl = s1 - s0, int(seq_lens[b])
        if ql == 0:
            continue
        nblk = (sl + bs - 1) // bs
        blocks = block_tables[b, :nblk].long()
        k = k_cache[blocks].permute(1, 0, 2, 3).reshape(hk, nblk * bs, d)[:, :sl].float()
        v = v_cache[blocks].permute(1, 0, 2, 3).reshape(hk, nblk * bs, d)[:, :sl].float()
        qq = q[s0:s1].float().view(ql, hk, g, d).permute(1, 2, 0, 3)  # [hk, g, ql, d]
        sc = torch.einsum("hgqd,hkd->hgqk", qq, k) * scale
        qpos = torch.arange(sl - ql, sl)
        kpos = torch.arange(sl)
        mask = kpos[None, :] > qpos[:, None]
        sc = sc.masked_fill(mask, float("-inf"))
        p = sc.softmax(-1)
        o = torch.einsum("hgqk,hkd->hgqd", p, v)  # [hk, g, ql, d]
        out[s0:s1] = o.permute(2, 0, 1, 3).reshape(ql, hq, d).to(q.dtype)
    return out


def silu_mul(x: torch.Tensor) -> torch.Tensor:
    f = x.shape[-1] // 2
    xf = x.float()
    return (torch.nn.functional.silu(xf[..., :f]) * xf[..., f:]).to(x.dtype)


def spec_verify(draft, target, seq_lens):
    """Greedy accept + commit. Returns (out_tokens, accept, next_token, new_seq_lens)."""
    b, k = draft.shape
    eq = (draft == target[:, :k]) & (draft >= 0)
    accept = torch.cumprod(eq.int(), dim=1).sum(1).int()
    out = torch.full((b, k + 1), -1, dtype=torch.long, device=draft.device)
    idx = torch.arange(k + 1, device=draft.device)
    keep = idx[None, :k] < accept[:, None].long()
    out[:, :k] = torch.where(keep, draft, out[:, :k])
    nxt = target.gather(1, accept.long()[:, None])[:, 0]
    out.scatter_(1, accept.long()[:, None], nxt[:, None])
    return out, accept, nxt, seq_lens + accept.long() + 1


# ----------------------------------------------------------------------------- Gated DeltaNet
def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    return xf / torch.sqrt((xf * xf).sum(-1, keepdim=True) + eps)


def gdn_gates(a: torch.Tensor, b: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor):
    """g = -exp(a_log) * softplus(a + dt_bias) (softplus(x) = x above 20), beta = sigmoid(b)."""
    x = a.float() + dt_bias.float()
    sp = torch.where(x > 20.0, x, torch.log1p(torch.exp(torch.clamp(x, max=20.0))))
    return -torch.exp(a_log.float()) * sp, torch.sigmoid(b.float())


def gdn_step(S: torch.Tensor, q, k, v, g, beta):
    """One recurrent step for all heads. S [HV, V, K] fp32 (updated in place); q,k [HV, K] (normed,
    q pre-scaled); v [HV, V]; g, beta [HV].  Returns o [HV, V]."""
    S.mul_(torch.exp(g)[:, None, None])
    sk = torch.einsum("hvk,hk->hv", S, k)
    vp = beta[:, None] * (v - sk)
    S.add_(vp[:, :, None] * k[:, None, :])
    return torch.einsum("hvk,hk->hv", S, q)


def gdn_conv(x: torch.Tensor, w: torch.Tensor, state: torch.Tensor):
    """Causal depthwise conv + SiLU over a token run. x [T, C], w [C, KW], state [C, KW-1]
    (the previous KW-1 inputs). Returns (y [T, C], new_state)."""
    kw = w.shape[1]
    xs = torch.cat([state.t().float(), x.float()], 0)  # [KW-1+T, C]
    T = x.shape[0]
    y = torch.zeros(T, x.shape[1], dtype=torch.float32)
    for j in range(kw):
        y += xs[j:j + T] * w[:, j].float()
    return torch.nn.functional.silu(y), xs[-(kw - 1):].t().contiguous()


def gated_rms_norm(o: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """rms_norm(o) over the last dim * w * silu(z)."""
    of = o.float()
    inv = torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps)
    return of * inv * w.float() * torch.nn.functional.silu(z.float())


def spec_advance(out_tokens, accept, next_token, seq_new, cand, clen, native, hyb_min: int):
    """Async-scheduling advance (restates the reference's device `resolve`, async_spec.py:102-120, for a
    candidate checked against this step's accepted tokens): returns (win [B, k+1], seq [B], real [B])."""
    B, W = out_tokens.shape[0], out_tokens.shape[1]
    k = W - 1
    win = torch.full((B, W), -1, dtype=torch.long)
    real = torch.zeros(B, dtype=torch.int32)
    for b in range(B):
        o = int(accept[b]) + 1
        cl = int(clen[b])
        aligned = o <= cl and all(int(cand[b, j]) == int(out_tokens[b, j]) for j in range(o))
        n_real = min(k, max(cl - o, 0)) if aligned else 0
        win[b, 0] = next_token[b]
        if native is not None and n_real < hyb_min:
            win[b, 1:] = native[b, :k]
        else:
            for j in range(n_real):
                win[b, 1 + j] = cand[b, o + j]
            real[b] = n_real
    return win, seq_new[:B].clone(), real


# ----------------------------------------------------------------------------- NVFP4
E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def nvfp4_global_scale(w: torch.Tensor) -> torch.Tensor:
    return (w.float().abs().max() / (6.0 * 448.0)).reshape(1).clamp_min(1e-12)


def nvfp4_quantize(w: torch.Tensor, global_scale: torch.Tensor):
    """(packed uint8 [N, K/2], scales e4m3 [N, K/16]) in the ModelOpt NVFP4 layout."""
    N, K = w.shape
    wf = w.float().view(N, K // 16, 16)
    g = float(global_scale.reshape(-1)[0])
    amax = wf.abs().amax(-1)
    sc = (amax / 6.0 / g).to(torch.float8_e4m3fn)
    s = sc.float() * g
    x = wf / torch.where(s > 0, s, torch.ones_like(s))[..., None]
    a = x.abs()
    mids = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    odd = torch.tensor([False, True, False, True, False, True, False])
    # nearest e2m1 magnitude; exact midpoints go to the even code
    code = ((a[..., None] > mids).sum(-1) + ((a[..., None] == mids) & odd).sum(-1)).to(torch.uint8)
    code = torch.where(x < 0, code | 8, code)  # negative values keep the sign bit (-0 included)
    code = code.view(N, K)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).to(torch.uint8)
    return packed.contiguous(), sc.contiguous()


def nvfp4_dequantize(packed: torch.Tensor, scales: torch.Tensor, global_scale: torch.Tensor) -> torch.Tensor:
    N = packed.shape[0]
    K = packed.shape[1] * 2
    lo = (packed & 15).long()
    hi = (packed >> 4).long()
    codes = torch.stack([lo, hi], -1).view(N, K)
    mag = E2M1[codes & 7]
    val = torch.where(codes & 8 > 0, -mag, mag)
    s = scales.float().repeat_interleave(16, dim=1) * float(global_scale.reshape(-1)[0])
    return (val * s).to(torch.bfloat16)


def e2m1_codes(x: torch.Tensor) -> torch.Tensor:
    """Nearest e2m1 code of each value (exact midpoints to the even code; bit 3 = sign, -0 included)."""
    a = x.abs()
    mids = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], device=x.device)
    odd = torch.tensor([False, True, False, True, False, True, False], device=x.device)
    code = ((a[..., None] > mids).sum(-1) + ((a[..., None] == mids) & odd).sum(-1)).to(torch.uint8)
    return torch.where(x < 0, code | 8, code)


def nvfp4_quant_act(x: torch.Tensor, static_g: float = 0.0):
    """NVFP4 quantisation of activations [R, K] with a per-row global multiplier g.

    g = static_g when given (the checkpoint's 1 / input_scale), else 2688 / amax(|row|) (1 for a zero
    row); block scale s = e4m3(amax16 * (g / 6)) (saturating at 448); code = e2m1(x * (g / s)).
    Returns (packed uint8 [R, K/2], scales uint8 (e4m3 bits) [R, K/16], a_scale fp32 [R] = 1 / g).
    Reference semantics: suffix_hybrid/helion_kernels/nvfp4_gemm.py:213-240 (`nvfp4_quant_act_body`,
    there with a static g)."""
    xf = x.float()
    R, K = xf.shape
    if static_g > 0:
        g = torch.full((R,), float(static_g), dtype=torch.float32, device=x.device)
    else:
        amax = xf.abs().amax(1)
        g = torch.where(amax > 0, torch.tensor(2688.0, device=x.device) / torch.where(amax > 0, amax, 1.0),
                        torch.ones_like(amax))
    g6 = g / 6.0
    blocks = xf.view(R, K // 16, 16)
    s = (blocks.abs().amax(-1) * g6[:, None]).clamp(max=448.0).to(torch.float8_e4m3fn)
    sf = s.float()
    inv = torch.where(sf > 0, g[:, None] / torch.where(sf > 0, sf, 1.0), torch.zeros_like(sf))
    code = e2m1_codes(blocks * inv[..., None]).view(R, K)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).to(torch.uint8)
    return packed.contiguous(), s.view(torch.uint8).contiguous(), 1.0 / g


def nvfp4_codes_value(packed: torch.Tensor) -> torch.Tensor:
    """e2m1 values [R, K] (fp32) of packed codes [R, K/2]."""
    R = packed.shape[0]
    lo = (packed & 15).long()
    hi = (packed >> 4).long()
    codes = torch.stack([lo, hi], -1).view(R, -1)
    mag = E2M1.to(packed.device)[codes & 7]
    return torch.where(codes & 8 > 0, -mag, mag)


def nvfp4_w4a4_linear(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, global_scale: torch.Tensor,
                      static_g: float = 0.0) -> torch.Tensor:
    """fp32 oracle of the block-scaled W4A4 GEMM: quantise x, then sum of dequantised products."""
    xq, xs, a_scale = nvfp4_quant_act(x, static_g)
    xa = nvfp4_codes_value(xq) * xs.view(torch.float8_e4m3fn).float().repeat_interleave(16, dim=1)
    wv = nvfp4_codes_value(packed) * scales.view(torch.uint8).view(torch.float8_e4m3fn).float().repeat_interleave(16, dim=1)
    return (xa @ wv.t()) * a_scale[:, None] * float(global_scale.reshape(-1)[0])


def e4m3_qdq(x: torch.Tensor) -> torch.Tensor:
    """Values rounded to e4m3 (nearest even, saturating at +-448), as fp32."""
    return x.float().clamp(-448.0, 448.0).to(torch.float8_e4m3fn).float()


def _mla_fp4_blocks(c: torch.Tensor):
    """Block scales (e4m3, [N, 16-value blocks]) and e2m1 codes ([N, Cl]) of latent rows c [N, Cl]:
    s = e4m3(max(amax16 / 6, 2^-9)), code = e2m1_rne(x * (1 / s))."""
    x = c.float().reshape(c.shape[0], -1, 16)
    s = (x.abs().amax(-1) / 6.0).clamp(2.0 ** -9, 448.0).to(torch.float8_e4m3fn)
    codes = e2m1_codes(x * (1.0 / s.float())[..., None])
    return s, codes.reshape(c.shape[0], -1)


def mla_fp4_qdq(c: torch.Tensor) -> torch.Tensor:
    """Latent values as the NVFP4 latent cache returns them (code * s, fp32)."""
    shape = c.shape
    s, codes = _mla_fp4_blocks(c.reshape(-1, shape[-1]))
    mag = E2M1.to(c.device)[(codes & 7).long()]
    val = torch.where(codes & 8 > 0, -mag, mag).view(codes.shape[0], -1, 16) * s.float()[..., None]
    return val.reshape(shape)


def mla_fp4_scale_pos(kv_lora: int) -> torch.Tensor:
    """Byte of block scale s inside the row's scale region: (kv_lora / 64) * (s % 4) + s // 4 (a bijection
    on the kv_lora / 16 scales; 8 * (s % 4) + s // 4 at kv_lora 512)."""
    s = torch.arange(kv_lora // 16)
    return (kv_lora // 64) * (s % 4) + s // 4


def mla_fp4_pack(c: torch.Tensor, kpe: torch.Tensor) -> torch.Tensor:
    """NVFP4 latent cache rows [N, row_bytes] (uint8) of latent c [N, Cl] and rope kpe [N, R]: e2m1 pairs
    (low nibble = even dim), the rope values in e4m3, the permuted block scales, zero padding to 16 bytes.
    The row of vLLM's nvfp4_ds_mla cache (reference: kernels-oxide/nvfp4_ds_mla/src/main.rs:11-20)."""
    N, Cl = c.shape
    R = kpe.shape[1]
    s, codes = _mla_fp4_blocks(c)
    rows = torch.zeros(N, (Cl // 2 + R + Cl // 16 + 15) // 16 * 16, dtype=torch.uint8)
    rows[:, :Cl // 2] = codes[:, 0::2] | (codes[:, 1::2] << 4)
    rows[:, Cl // 2:Cl // 2 + R] = e4m3_qdq(kpe).to(torch.float8_e4m3fn).view(torch.uint8)
    rows[:, Cl // 2 + R + mla_fp4_scale_pos(Cl)] = s.view(torch.uint8)
    return rows


def mla_fp4_unpack(rows: torch.Tensor, kv_lora: int, rope: int) -> torch.Tensor:
    """Values [N, kv_lora + rope] (fp32) that NVFP4 latent rows hold."""
    N = rows.shape[0]
    codes = torch.stack([rows[:, :kv_lora // 2] & 15, rows[:, :kv_lora // 2] >> 4], -1).view(N, kv_lora).long()
    mag = E2M1[codes & 7]
    base = kv_lora // 2 + rope
    s = rows[:, base + mla_fp4_scale_pos(kv_lora)].contiguous().view(torch.float8_e4m3fn).float()
    lat = (torch.where(codes & 8 > 0, -mag, mag).view(N, -1, 16) * s[..., None]).view(N, kv_lora)
    pe = rows[:, kv_lora // 2:base].contiguous().view(torch.float8_e4m3fn).float()
    return torch.cat([lat, pe], -1)


# ----------------------------------------------------------------------------- MXFP8 (W8A8, block 32)
def mxfp8_quantize(x: torch.Tensor):
    """e4m3 codes (uint8 bits) [R, K] and ue8m0 scales [R, K/32]: s = 2^e with the smallest e keeping
    amax32 / s <= 448, code = e4m3(x / s) (exact power-of-two scaling, round to nearest even)."""
    R, K = x.shape
    xf = x.float().view(R, K // 32, 32)
    am = xf.abs().amax(-1)
    m, ex = torch.frexp(am / 448.0)
    e = torch.where(m == 0.5, ex - 1, ex)
    e = torch.where(am > 0, e, torch.full_like(e, -127)).clamp(-127, 127)
    codes = (xf * torch.pow(2.0, -e.float())[..., None]).to(torch.float8_e4m3fn)
    return codes.view(torch.uint8).view(R, K).contiguous(), (e + 127).to(torch.uint8).contiguous()


def mxfp8_dequantize(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    R, K = codes.shape
    v = codes.view(torch.float8_e4m3fn).float().view(R, K // 32, 32)
    return (v * torch.pow(2.0, scales.float() - 127.0)[..., None]).view(R, K)


def mxfp8_linear(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 oracle of the MXFP8 W8A8 GEMM: quantise x like the kernel, sum dequantised products."""
    xc, xs = mxfp8_quantize(x)
    return mxfp8_dequantize(xc, xs) @ mxfp8_dequantize(codes, scales).t()


# ----------------------------------------------------------------------------- MLA / DSA
def mla_attention(q_lat, q_pe, latent, block_tables, seq_lens, q_start, scale, kv_lora, topk=None):
    """Absorbed MLA over a latent cache [blocks, bs, kv_lora + rope].

    q_lat [T, H, kv_lora], q_pe [T, H, rope]; returns o_lat [T, H, kv_lora] (fp32).
    topk [T, K] (absolute positions, -1 = unused) restricts each query to those keys (DSA)."""
    bs = latent.shape[1]
    T, H, _ = q_lat.shape
    out = torch.zeros(T, H, kv_lora, dtype=torch.float32, device=q_lat.device)
    for b in range(seq_lens.shape[0]):
        s0, s1 = int(q_start[b]), int(q_start[b + 1])
        ql, sl = s1 - s0, int(seq_lens[b])
        if ql == 0:
            continue
        nblk = (sl + bs - 1) // bs
        C = latent[block_tables[b, :nblk].long()].reshape(nblk * bs, -1)[:sl].float()
        sc = (torch.einsum("thc,sc->ths", q_lat[s0:s1].float(), C[:, :kv_lora]) +
              torch.einsum("thr,sr->ths", q_pe[s0:s1].float(), C[:, kv_lora:])) * scale
        qpos = torch.arange(sl - ql, sl, device=q_lat.device)
        mask = torch.arange(sl, device=q_lat.device)[None, :] > qpos[:, None]
        if topk is not None:
            sel = torch.zeros(ql, sl + 1, dtype=torch.bool, device=q_lat.device)
            idx = topk[s0:s1].long().clamp(-1, sl - 1)
            sel.scatter_(1, torch.where(idx < 0, torch.full_like(idx, sl), idx), True)
            mask = mask | ~sel[:, :sl]
        sc = sc.masked_fill(mask[:, None, :], float("-inf"))
        out[s0:s1] = torch.einsum("ths,sc->thc", sc.softmax(-1), C[:, :kv_lora])
    return out


DSA_PAGE_KEYS, DSA_DIM = 64, 128
DSA_KEY_BYTES = DSA_PAGE_KEYS * DSA_DIM  # key bytes of a page; the 64 f32 scales follow


def dsa_quant(x):
    """Per-row e4m3 quantisation of [..., 128] values: s = amax / 448 (1 for a zero row), codes = e4m3(x / s)
    rounded to nearest even.  Returns (codes as float32, s [..., 1])."""
    x = x.float()
    am = x.abs().amax(-1, keepdim=True)
    s = torch.where(am > 0, am / 448.0, torch.ones_like(am))
    return (x / s).to(torch.float8_e4m3fn).float(), s


def dsa_cache_write(cache, k, slots):
    """Write keys into the indexer page cache ([pages, 8448] uint8): page slot // 64, row slot % 64."""
    ok = slots >= 0
    if not bool(ok.any()):
        return
    x = k[ok].float()
    s_all = slots[ok].long()
    codes, sc = dsa_quant(x)
    cb = codes.to(torch.float8_e4m3fn).view(torch.uint8)
    sb = sc[:, 0].contiguous().view(torch.uint8).view(-1, 4)
    pg, r = s_all // DSA_PAGE_KEYS, s_all % DSA_PAGE_KEYS
    cols = torch.arange(DSA_DIM, device=cache.device)
    cache[pg[:, None], (r * DSA_DIM)[:, None] + cols[None]] = cb
    c4 = torch.arange(4, device=cache.device)
    cache[pg[:, None], (DSA_KEY_BYTES + r * 4)[:, None] + c4[None]] = sb


def dsa_keys(cache):
    """Dequantised keys [pages, 64, 128] (e4m3 codes) and scales [pages, 64] of the indexer page cache."""
    keys = cache[:, :DSA_KEY_BYTES].contiguous().view(torch.float8_e4m3fn).float().view(-1, DSA_PAGE_KEYS, DSA_DIM)
    scales = cache[:, DSA_KEY_BYTES:].contiguous().view(torch.float32).view(-1, DSA_PAGE_KEYS)
    return keys, scales


def dsa_logits(qi, w, kcache, block_tables, seq_lens, q_start):
    """Per-token indexer logits over the causal keys: logits[t][p] = ks[p] * sum_h relu(q8[t,h] . k8[p]) *
    w[t,h] * qs[t,h] (fp32, float64 accumulation), one tensor per query token."""
    keys, ks = dsa_keys(kcache)
    q8, qs = dsa_quant(qi)
    wq = w.float() * qs[..., 0]
    out = []
    for b in range(seq_lens.shape[0]):
        s0, s1 = int(q_start[b]), int(q_start[b + 1])
        ql, sl = s1 - s0, int(seq_lens[b])
        if ql == 0:
            continue
        nblk = (sl + DSA_PAGE_KEYS - 1) // DSA_PAGE_KEYS
        pages = block_tables[b, :nblk].long()
        Kc = keys[pages].reshape(-1, DSA_DIM)[:sl].double()
        KS = ks[pages].reshape(-1)[:sl].double()
        lg = (torch.relu(torch.einsum("thd,sd->ths", q8[s0:s1].double(), Kc)) * wq[s0:s1].double()[..., None]).sum(1)
        lg = lg * KS[None]
        for j in range(ql):
            out.append(lg[j, : sl - ql + j + 1].float())
    return out


def dsa_topk(qi, w, kcache, block_tables, seq_lens, q_start, k):
    """Lightning indexer over the fp8 page cache: the k largest causal logits per query token, positions in
    ascending order, -1 padded ([T, k] int32).  Equal logits prefer the later position."""
    T = qi.shape[0]
    out = torch.full((T, k), -1, dtype=torch.int32, device=qi.device)
    for t, lg in enumerate(dsa_logits(qi, w, kcache, block_tables, seq_lens, q_start)):
        n = lg.shape[0]
        if n <= k:
            out[t, :n] = torch.arange(n, dtype=torch.int32)
            continue
        # stable sort of the reversed row: among equal logits the later position comes first
        idx = torch.sort(lg.flip(-1), descending=True, stable=True).indices[:k]
        out[t] = torch.sort(n - 1 - idx).values.to(torch.int32)
    return out
