"""Differentiable replay of the one-layer draft head (models/llama.py DraftHead, eagle or mtp style).

Serving runs the head through paged-attention kernels without autograd; training and gating replay the
same math in plain torch over a token sequence: at position p the head reads the target's pre-norm
hidden state pre[p] and the token S[p+1] and predicts S[p+2].  Frozen weights stay in the model dtype;
the adapters given in `ad` ({linear name: (A, B, scale)}) are added like Linear.lora.  Under tensor
parallelism each rank runs its shard with the autograd collectives of tune/collectives.py, so the
replay reduces exactly where serving does.

`teacher_forced` returns logits and the per-position keys/values and pre-norm outputs; `chain_accept`
replays the greedy draft chain (depths 1..k, the head's own pre-norm output as the next feature) from
anchor positions and returns how many drafts the true continuation accepts at each anchor.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
import torch.nn.functional as F

from ..ops import reference as ref
from .collectives import copy_to_tp, gather_from_tp, reduce_from_tp

TARGETS = ("qkv", "o", "gate_up", "down")


def linears(draft) -> Dict[str, object]:
    L = draft.layer
    return {"qkv": L.attn.qkv, "o": L.attn.o, "gate_up": L.mlp.gate_up, "down": L.mlp.down}


def _lin(x: torch.Tensor, lin, ad) -> torch.Tensor:
    y = F.linear(x.to(lin.weight.dtype), lin.weight).float()
    if ad is not None:
        a, b, scale = ad
        y = y + scale * ((x.float() @ a.float().t()) @ b.float().t())
    return y


def _rms(x, w, eps):
    return ref.rms_norm(x.float(), w, eps).float()


class _Fwd:
    def __init__(self, draft, ad: Optional[dict]):
        self.d, self.ad = draft, ad or {}
        self.L = draft.layer
        self.A = draft.layer.attn
        self.eps = draft.cfg.norm_eps
        self.lin = linears(draft)

    def inputs(self, tokens, feats):
        d = self.d
        e = d.target.embed[tokens].float()
        f = feats.float()
        if d.style == "mtp":
            e = _rms(e, d.enorm.weight, d.enorm.eps)
            f = _rms(f, d.hnorm.weight, d.hnorm.eps)
        return F.linear(torch.cat([e, f], -1).to(d.fc.dtype), d.fc).float()

    def qkv(self, residual, positions):
        A = self.A
        x = copy_to_tp(_rms(residual, self.L.input_norm.weight, self.eps))
        qkv = _lin(x, self.lin["qkv"], self.ad.get("qkv"))
        t = qkv.shape[0]
        q = qkv[:, : A.hq * A.d].view(t, A.hq, A.d)
        k = qkv[:, A.hq * A.d:(A.hq + A.hk) * A.d].view(t, A.hk, A.d)
        v = qkv[:, (A.hq + A.hk) * A.d:].view(t, A.hk, A.d)
        return ref.apply_rope(q, positions, A.cos_sin), ref.apply_rope(k, positions, A.cos_sin), v

    def post(self, residual, attn):
        o = reduce_from_tp(_lin(attn.reshape(attn.shape[0], -1), self.lin["o"], self.ad.get("o")))
        residual = residual + o
        h = copy_to_tp(_rms(residual, self.L.post_norm.weight, self.L.post_norm.eps))
        gu = _lin(h, self.lin["gate_up"], self.ad.get("gate_up"))
        g, u = gu.chunk(2, dim=-1)
        m = reduce_from_tp(_lin(F.silu(g) * u, self.lin["down"], self.ad.get("down")))
        residual = residual + m
        return _rms(residual, self.d.norm.weight, self.d.norm.eps), residual

    def logits(self, normed):
        lm = self.d.target.lm_head
        return gather_from_tp(F.linear(copy_to_tp(normed).to(lm.weight.dtype), lm.weight).float())


def teacher_forced(draft, ad, tokens: torch.Tensor, feats: torch.Tensor, positions: torch.Tensor):
    """tokens / feats / positions [T] ... -> (logits [T, V], k [T, hk, d], v [T, hk, d], pre-norm out [T, H])."""
    fw = _Fwd(draft, ad)
    residual = fw.inputs(tokens, feats)
    q, k, v = fw.qkv(residual, positions)
    A = fw.A
    g = A.hq // A.hk
    kk = k.repeat_interleave(g, dim=1).transpose(0, 1)  # [hq, T, d]
    vv = v.repeat_interleave(g, dim=1).transpose(0, 1)
    attn = F.scaled_dot_product_attention(q.transpose(0, 1).unsqueeze(0), kk.unsqueeze(0), vv.unsqueeze(0),
                                          is_causal=True, scale=A.scale)[0].transpose(0, 1)
    normed, out = fw.post(residual, attn)
    return fw.logits(normed), k, v, out


@torch.no_grad()
def chain_accept(draft, ad, seq: torch.Tensor, feats: torch.Tensor, anchors: torch.Tensor, k: int,
                 return_tokens: bool = False):
    """Accepted draft length at each anchor p (drafts S[p+2..p+k+1] proposed from pre[p], S[p+1]); with
    return_tokens also the full drafted chains [anchors, k] (the chain runs all k depths then).

    Depth 1 is the teacher-forced row p; depth s >= 2 feeds the previous draft token and the head's own
    pre-norm output at position p+s-1 and attends to the teacher-forced rows <= p plus the chain's rows."""
    n = seq.shape[0] - 1  # draft rows 0..n-1 read (pre[p], S[p+1])
    pos = torch.arange(n, device=seq.device)
    logits, k_tf, v_tf, out_tf = teacher_forced(draft, ad, seq[1:n + 1], feats[:n], pos)
    fw = _Fwd(draft, ad)
    A = fw.A
    g = A.hq // A.hk
    na = anchors.shape[0]
    tok = logits[anchors].argmax(-1)
    feat = out_tf[anchors]
    alive = torch.ones(na, dtype=torch.bool, device=seq.device)
    acc = torch.zeros(na, dtype=torch.long, device=seq.device)
    drafted = []
    ck, cv = [], []
    for s in range(1, k + 1):
        drafted.append(tok)
        tgt_idx = anchors + s + 1
        ok = tgt_idx < seq.shape[0]
        hit = alive & ok & (tok == seq[tgt_idx.clamp(max=seq.shape[0] - 1)])
        acc += hit.long()
        alive = hit
        if s == k or (not bool(alive.any()) and not return_tokens):
            break
        # next chain step: position p + s, input (draft token, own pre-norm output)
        residual = fw.inputs(tok, feat)
        q, kn, vn = fw.qkv(residual, anchors + s)
        ck.append(kn)
        cv.append(vn)
        qh = q  # [na, hq, d]
        sc_tf = torch.einsum("ahd,thd->aht", qh, k_tf.repeat_interleave(g, dim=1)) * A.scale
        mask = pos[None, None, :] > anchors[:, None, None]
        sc_tf = sc_tf.masked_fill(mask, float("-inf"))
        kc = torch.stack(ck, 1).repeat_interleave(g, dim=2)  # [na, s, hq, d]
        vc = torch.stack(cv, 1).repeat_interleave(g, dim=2)
        sc_ch = torch.einsum("ahd,ashd->ahs", qh, kc) * A.scale
        p_all = torch.softmax(torch.cat([sc_tf, sc_ch], -1), -1)
        attn = torch.einsum("aht,thd->ahd", p_all[..., :n], v_tf.repeat_interleave(g, dim=1)) + \
            torch.einsum("ahs,ashd->ahd", p_all[..., n:], vc)
        normed, feat = fw.post(residual, attn)
        tok = fw.logits(normed).argmax(-1)
    if return_tokens:
        return acc, torch.stack(drafted, 1)
    return acc


def train_loss(draft, ad, seq: torch.Tensor, feats: torch.Tensor, start: int = 0) -> Tuple[torch.Tensor, int]:
    """Depth-1 teacher-forced cross-entropy of the head over one sequence (rows >= start count)."""
    n = seq.shape[0] - 2
    if n <= start:
        return None, 0
    pos = torch.arange(n + 0, device=seq.device)
    logits, _, _, _ = teacher_forced(draft, ad, seq[1:n + 1], feats[:n], pos)
    loss = F.cross_entropy(logits[start:], seq[start + 2:n + 2])
    return loss, n - start


# ---------------------------------------------------------------------------------------- target model
def layer_linears(layer, prefix: str) -> Dict[str, object]:
    return {prefix + "qkv": layer.attn.qkv, prefix + "o": layer.attn.o, prefix + "gate_up": layer.mlp.gate_up,
            prefix + "down": layer.mlp.down}


def target_linears(model) -> Dict[str, object]:
    out = {}
    for i, L in enumerate(model.layers):
        out.update(layer_linears(L, f"layers.{i}."))
    return out


def _layer(L, ad: dict, prefix: str, residual: torch.Tensor, positions: torch.Tensor, eps: float) -> torch.Tensor:
    """One decoder layer (models/common.py DecoderLayer) on the residual stream, causal over the sequence."""
    A = L.attn
    x = copy_to_tp(_rms(residual, L.input_norm.weight, eps))
    qkv = _lin(x, A.qkv, ad.get(prefix + "qkv"))
    t = qkv.shape[0]
    q = ref.apply_rope(qkv[:, : A.hq * A.d].view(t, A.hq, A.d), positions, A.cos_sin)
    k = ref.apply_rope(qkv[:, A.hq * A.d:(A.hq + A.hk) * A.d].view(t, A.hk, A.d), positions, A.cos_sin)
    v = qkv[:, (A.hq + A.hk) * A.d:].view(t, A.hk, A.d)
    g = A.hq // A.hk
    attn = F.scaled_dot_product_attention(q.transpose(0, 1).unsqueeze(0),
                                          k.repeat_interleave(g, dim=1).transpose(0, 1).unsqueeze(0),
                                          v.repeat_interleave(g, dim=1).transpose(0, 1).unsqueeze(0),
                                          is_causal=True, scale=A.scale)[0].transpose(0, 1)
    residual = residual + reduce_from_tp(_lin(attn.reshape(t, -1), A.o, ad.get(prefix + "o")))
    h = copy_to_tp(_rms(residual, L.post_norm.weight, L.post_norm.eps))
    gu = _lin(h, L.mlp.gate_up, ad.get(prefix + "gate_up"))
    gg, u = gu.chunk(2, dim=-1)
    return residual + reduce_from_tp(_lin(F.silu(gg) * u, L.mlp.down, ad.get(prefix + "down")))


def target_logits(model, ad: Optional[dict], tokens: torch.Tensor, checkpoint: bool = True) -> torch.Tensor:
    """Full target forward (Llama family) over one sequence: logits [T, V] (vocab gathered under TP).
    checkpoint recomputes each layer in the backward pass (activation memory of one layer)."""
    ad = ad or {}
    eps = model.cfg.norm_eps
    positions = torch.arange(tokens.shape[0], device=tokens.device)
    residual = model.embed[tokens].float()
    for i, L in enumerate(model.layers):
        fn = lambda r, L=L, i=i: _layer(L, ad, f"layers.{i}.", r, positions, eps)
        if checkpoint and residual.requires_grad:
            residual = torch.utils.checkpoint.checkpoint(fn, residual, use_reentrant=False)
        else:
            residual = fn(residual)
    normed = _rms(residual, model.norm.weight, model.norm.eps)
    lm = model.lm_head
    return gather_from_tp(F.linear(copy_to_tp(normed).to(lm.weight.dtype), lm.weight).float())
