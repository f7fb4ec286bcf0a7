"""Model runner: prefill and the fused verify + draft decode step.

Decode step for a batch of B requests, each with a verify window
[t_prev, d_1..d_k] at positions L..L+k (L = committed cache length):

  1. target forward over the B*(k+1) window tokens (writes their KV);
  2. greedy target tokens (vocab-parallel argmax, no logits gather);
  3. spec_verify kernel: accept run, emitted tokens, bonus, L += a + 1;
  4. draft pass 1 over the same window (features = target pre-norm hidden,
     tokens = the verified next tokens) -> first native draft from row a;
  5. k-1 single-token draft steps -> native drafts [B, k].

Everything after the host upload is static-shape per (batch bucket, verify
width), so the whole step is captured once per pair as a CUDA graph and
replayed.  The verify width W of a step is 1 + the longest draft any row
publishes (at most k + 1): when every row's drafts are short -- suffix-only
or n-gram misses, EWMA-gated widths -- the step verifies fewer tokens per
row, and a step with no drafts at all is a plain 1-token decode (reference
behaviour: ragged widths, width-0 rows cost a plain decode,
suffix_hybrid/wrap_v2.py:1503-1569).  Rows with fewer drafts than W - 1 are
padded with -1, which never matches a target token.  Padded rows of a
bucket point at the reserved scratch block 0.
"""
from __future__ import annotations

import math
import os
from typing import Dict, List, Optional

import numpy as np
import torch

from .. import ops
from ..models.common import AttnMeta
from .kv_cache import blocks_for

BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256)


def _max_rows(rows: int) -> int:
    """Query rows per attention tile the kernel is specialised for (it picks its in-CTA key split from this).
    Batch-invariant mode always reports a full tile, so the key split -- which changes the softmax merge
    order -- does not depend on the verify width."""
    if os.environ.get("SH_BATCH_INVARIANT", "0") == "1":
        return 64
    return min(64, rows)


def bucket_for(n: int, max_batch: int) -> int:
    for b in BUCKETS:
        if b >= n and b <= max_batch:
            return b
    return max_batch


class Runner:
    def __init__(self, model, draft, caches, draft_caches, k: int, max_batch: int, max_blocks: int,
                 block_size: int, device, use_graphs: bool):
        self.model, self.draft = model, draft
        self.caches, self.dcaches = caches, draft_caches
        self.k = k
        self.W = k + 1
        self.max_batch = max_batch
        self.max_blocks = max_blocks
        self.bs = block_size
        self.device = device
        self.use_graphs = use_graphs and torch.device(device).type == "cuda"
        self.group = model.cfg.heads // model.cfg.kv_heads
        B, W = max_batch, self.W
        L = dict(dtype=torch.long, device=device)
        # Static device inputs / outputs of the decode step.
        self.win = torch.zeros(B, W, **L)
        self.seq = torch.zeros(B, **L)  # committed length L before the window
        self.bt = torch.zeros(B, max_blocks, dtype=torch.int32, device=device)
        self.target = torch.zeros(B, W, **L)
        self.out_tokens = torch.zeros(B, W, **L)
        self.accept = torch.zeros(B, dtype=torch.int32, device=device)
        self.next_tok = torch.zeros(B, **L)
        self.native = torch.zeros(B, max(k, 1), **L)
        self.seq_new = torch.zeros(B, **L)
        self.slots = torch.zeros(B, **L)  # recurrent-state slot per row (0 = scratch)
        self.pending = torch.zeros(max_batch + 1, dtype=torch.int32, device=device)
        self.recurrent = bool(getattr(model, "has_recurrent_state", False))
        self.ar_w = torch.arange(W, **L)
        self.ar_b = torch.arange(B, **L)
        pin = torch.device(device).type == "cuda"
        # Pinned host staging (H2D inputs, D2H results).
        self.h_win = torch.zeros(B, W, dtype=torch.long, pin_memory=pin)
        self.h_seq = torch.zeros(B, dtype=torch.long, pin_memory=pin)
        self.h_bt = torch.zeros(B, max_blocks, dtype=torch.int32, pin_memory=pin)
        self.h_out = torch.zeros(B, W, dtype=torch.long, pin_memory=pin)
        self.h_acc = torch.zeros(B, dtype=torch.int32, pin_memory=pin)
        self.h_nat = torch.zeros(B, max(k, 1), dtype=torch.long, pin_memory=pin)
        self.h_slots = torch.zeros(B, dtype=torch.long, pin_memory=pin)
        self._tiles: Dict[tuple, tuple] = {}
        self.graphs: Dict[tuple, torch.cuda.CUDAGraph] = {}  # (bucket, verify width) -> graph
        self.event = torch.cuda.Event() if pin else None
        # Device time of the last decode step (H2D of its inputs .. D2H of its results).
        self.ev0 = torch.cuda.Event(enable_timing=True) if pin else None
        self.ev1 = torch.cuda.Event(enable_timing=True) if pin else None
        self.last_device_ms = 0.0
        self.last_width = self.W
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self._async = None  # buffers of the pipelined (async-scheduling) step, made on first use

    # ------------------------------------------------------------------ async scheduling
    def _async_buffers(self, cand_len: int):
        """Parity-double-buffered pinned staging + device candidate buffers of the pipelined step."""
        if self._async is not None and self._async["L"] == cand_len:
            return self._async
        B, W, pin = self.max_batch, self.W, torch.device(self.device).type == "cuda"
        P = lambda *shape, dt=torch.long: [torch.zeros(*shape, dtype=dt, pin_memory=pin) for _ in range(2)]
        self._async = dict(
            L=cand_len, h_win=P(B, W), h_seq=P(B), h_bt=P(B, self.max_blocks, dt=torch.int32), h_slots=P(B),
            h_cand=P(B, cand_len), h_clen=P(B, dt=torch.int32), h_out=P(B, W), h_acc=P(B, dt=torch.int32),
            h_nat=P(B, max(self.k, 1)), h_used=P(B, W), h_real=P(B, dt=torch.int32),
            cand=torch.zeros(B, cand_len, dtype=torch.long, device=self.device),
            clen=torch.zeros(B, dtype=torch.int32, device=self.device),
            real=torch.zeros(B, dtype=torch.int32, device=self.device),
            ev=[torch.cuda.Event() if pin else None for _ in range(2)], nb=None)
        return self._async

    def launch(self, parity: int, nb_real: int, bt: np.ndarray, slots: np.ndarray, win: np.ndarray = None,
               seq: np.ndarray = None, cand: np.ndarray = None, clen: np.ndarray = None, hyb_min: int = 0,
               cand_len: int = 1) -> None:
        """Enqueue one decode step without waiting for it (async scheduling).

        win/seq given: the window comes from the host (pipeline start).  Otherwise the window is built on
        the device by `spec_advance` from the previous launch's results (same rows, same bucket) and the
        host candidates cand [n, cand_len] / clen [n] computed one step earlier.  Results land in the
        parity's pinned buffers; `collect(parity)` waits for them.  Staging is double-buffered by parity:
        a parity is reused only after its previous step was collected.
        """
        A = self._async_buffers(cand_len)
        nb = bucket_for(nb_real, self.max_batch)
        if win is None and A["nb"] != nb:
            raise RuntimeError("device-advanced launch needs the previous launch's bucket")
        A["nb"] = nb
        nbt = self.max_blocks
        A["h_bt"][parity][:nb_real, : bt.shape[1]].numpy()[:] = bt
        A["h_bt"][parity][nb_real:nb] = 0
        A["h_slots"][parity][:nb_real].numpy()[:] = slots
        A["h_slots"][parity][nb_real:nb] = 0
        self.bt[:nb, :nbt].copy_(A["h_bt"][parity][:nb, :nbt], non_blocking=True)
        self.slots[:nb].copy_(A["h_slots"][parity][:nb], non_blocking=True)
        if win is not None:
            A["h_win"][parity][:nb_real].numpy()[:] = win
            A["h_seq"][parity][:nb_real].numpy()[:] = seq
            A["h_win"][parity][nb_real:nb] = 0
            A["h_seq"][parity][nb_real:nb] = 0
            self.win[:nb].copy_(A["h_win"][parity][:nb], non_blocking=True)
            self.seq[:nb].copy_(A["h_seq"][parity][:nb], non_blocking=True)
            A["real"][:nb].zero_()
        else:
            A["h_cand"][parity][:nb_real].numpy()[:] = cand
            A["h_clen"][parity][:nb_real].numpy()[:] = clen
            A["cand"][:nb].copy_(A["h_cand"][parity][:nb], non_blocking=True)
            A["clen"][:nb].copy_(A["h_clen"][parity][:nb], non_blocking=True)
            nat = self.native[:nb] if (self.draft is not None and self.k > 0 and hyb_min > 0) else None
            ops.spec_advance(self.out_tokens[:nb], self.accept[:nb], self.next_tok[:nb], self.seq_new[:nb],
                             A["cand"][:nb], A["clen"][:nb], nat, self.win[:nb], self.seq[:nb], A["real"][:nb],
                             hyb_min, nb_real)
        A["h_used"][parity][:nb].copy_(self.win[:nb], non_blocking=True)
        A["h_real"][parity][:nb].copy_(A["real"][:nb], non_blocking=True)
        if self.use_graphs:
            g = self.graphs.get((nb, self.W))
            if g is None:
                raise RuntimeError("capture the bucket's graph with a synchronous step first")
            g.replay()
        else:
            self._decode_body(nb)
        A["h_out"][parity][:nb].copy_(self.out_tokens[:nb], non_blocking=True)
        A["h_acc"][parity][:nb].copy_(self.accept[:nb], non_blocking=True)
        if self.draft is not None and self.k > 0:
            A["h_nat"][parity][:nb].copy_(self.native[:nb], non_blocking=True)
        if A["ev"][parity] is not None:
            A["ev"][parity].record()
        self.h2d_bytes = nb * (self.max_blocks * 4 + 8) + (nb * (self.W * 8 + 8) if win is not None
                                                           else nb * (cand_len * 8 + 4))
        self.d2h_bytes = nb * (2 * self.W * 8 + 8 + (self.k * 8 if self.draft is not None and self.k > 0 else 0))

    def collect(self, parity: int, nb_real: int):
        """Wait for a launched step; host views (out_tokens, accept, native, window used, real drafts)."""
        A = self._async
        if A["ev"][parity] is not None:
            A["ev"][parity].synchronize()
        return (A["h_out"][parity][:nb_real].numpy(), A["h_acc"][parity][:nb_real].numpy(),
                A["h_nat"][parity][:nb_real].numpy(), A["h_used"][parity][:nb_real].numpy(),
                A["h_real"][parity][:nb_real].numpy())

    def has_graph(self, nb_real: int) -> bool:
        return not self.use_graphs or (bucket_for(nb_real, self.max_batch), self.W) in self.graphs

    # ------------------------------------------------------------------ helpers
    def _tile_tensors(self, nb: int, qlen: int):
        key = (nb, qlen)
        if key not in self._tiles:
            req, row0 = ops.plan_attention_tiles([qlen] * nb, self.group // max(1, 1))
            qs = torch.arange(nb + 1, dtype=torch.long, device=self.device) * qlen
            self._tiles[key] = (torch.tensor(req, dtype=torch.int32, device=self.device),
                                torch.tensor(row0, dtype=torch.int32, device=self.device), qs)
        return self._tiles[key]

    def _slots(self, bt: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """pos [B, n] -> cache slots via the block table."""
        blk = bt.long().gather(1, torch.div(pos, self.bs, rounding_mode="floor"))
        return blk * self.bs + pos % self.bs

    def _meta(self, nb: int, qlen: int, pos: torch.Tensor, bt: torch.Tensor, seq_lens: torch.Tensor) -> AttnMeta:
        tr, t0, qs = self._tile_tensors(nb, qlen)
        kvh = self.model.kv_heads_local
        nsplit = ops.attention_splits(tr.numel(), kvh, self.max_blocks)
        return AttnMeta(positions=pos.reshape(-1), slot_mapping=self._slots(bt, pos).reshape(-1), block_tables=bt,
                        seq_lens=seq_lens, q_start=qs, tile_req=tr, tile_row0=t0, num_tokens=nb * qlen,
                        nsplit=nsplit, max_rows=_max_rows(qlen * self.group))

    def _draft_steps(self, d1: torch.Tensor, f1: torch.Tensor, lnew: torch.Tensor, bt: torch.Tensor, nb: int):
        """Draft tokens 2..k at positions lnew + s - 2 (s = 2..k)."""
        drafts = [d1]
        d, f = d1, f1
        for s in range(2, self.k + 1):
            pos = (lnew + (s - 2))[:, None]
            meta = self._meta(nb, 1, pos, bt, pos[:, 0] + 1)
            h, f = self.draft.forward(d, f, meta, self.dcaches)
            d = self.model.greedy(h)
            drafts.append(d)
        return torch.stack(drafts, 1)

    # ------------------------------------------------------------------ decode
    def _decode_body(self, nb: int, W: Optional[int] = None) -> None:
        W = self.W if W is None else W
        win, L, bt = self.win[:nb, :W], self.seq[:nb], self.bt[:nb]
        pos = L[:, None] + self.ar_w[None, :W]
        meta = self._meta(nb, W, pos, bt, L + W)
        meta.state_slots, meta.pending, meta.window = self.slots[:nb], self.pending, W
        # win is a column slice of the static [B, k + 1] buffer: copy it into one contiguous id vector
        # (for W = 1 a reshape would return a strided view, which the embedding kernel must not get).
        hid, pre = self.model.forward(win.contiguous().view(-1), meta, self.caches)
        target = self.target[:nb, :W]
        target.copy_(self.model.greedy(hid).view(nb, W))
        lnew = self.seq_new[:nb]
        lnew.copy_(L)
        if W > 1:
            ops.spec_verify(win[:, 1:], target, lnew, self.out_tokens[:nb, :W], self.accept[:nb], self.next_tok[:nb])
        else:
            self.out_tokens[:nb, :1].copy_(target)
            self.accept[:nb].zero_()
            self.next_tok[:nb].copy_(target[:, 0])
            lnew.add_(1)
        if self.recurrent:  # deferred commit: the next window replays accept+1 records
            self.pending.index_copy_(0, self.slots[:nb], (self.accept[:nb] + 1).to(torch.int32))
        if self.draft is not None and self.k > 0:
            tok_in = self.out_tokens[:nb, :W].clamp_min(0)
            dh, dpre = self.draft.forward(tok_in.reshape(-1), pre, meta, self.dcaches)
            sel = self.ar_b[:nb] * W + self.accept[:nb].long()
            d1 = self.model.greedy(dh.index_select(0, sel))
            f1 = dpre.index_select(0, sel)
            self.native[:nb].copy_(self._draft_steps(d1, f1, lnew, bt, nb))

    def decode(self, nb_real: int, win: np.ndarray, seq: np.ndarray, bt: np.ndarray, slots: np.ndarray = None,
               nb_min: int = 0, width: Optional[int] = None):
        """Run one decode step; returns host views (out_tokens, accept, native).  nb_min raises the batch
        bucket (data-parallel ranks run the same bucket; rows past nb_real are scratch padding).  width:
        the step's verify width (1..k+1, default k+1); win columns past it are not read."""
        nb = bucket_for(max(nb_real, nb_min, 1), self.max_batch)
        W = self.W if width is None else int(width)
        if not 1 <= W <= self.W:
            raise ValueError(f"verify width {W} outside 1..{self.W}")
        self.h_win[:nb_real].numpy()[:] = win
        self.h_seq[:nb_real].numpy()[:] = seq
        self.h_bt[:nb_real].numpy()[:, :bt.shape[1]] = bt
        self.h_slots[:nb_real].numpy()[:] = slots if slots is not None else 0
        if nb > nb_real:  # padded rows: scratch block 0 and scratch state slot 0
            self.h_win[nb_real:nb] = 0
            self.h_seq[nb_real:nb] = 0
            self.h_bt[nb_real:nb] = 0
            self.h_slots[nb_real:nb] = 0
        nbt = self.max_blocks
        if self.ev0 is not None:
            self.ev0.record()
        self.win[:nb].copy_(self.h_win[:nb], non_blocking=True)
        self.seq[:nb].copy_(self.h_seq[:nb], non_blocking=True)
        self.bt[:nb, :nbt].copy_(self.h_bt[:nb, :nbt], non_blocking=True)
        self.slots[:nb].copy_(self.h_slots[:nb], non_blocking=True)
        if self.use_graphs:
            g = self.graphs.get((nb, W))
            if g is None:
                g = self._capture(nb, W)
            g.replay()
        else:
            self._decode_body(nb, W)
        self.h_out[:nb].copy_(self.out_tokens[:nb], non_blocking=True)
        self.h_acc[:nb].copy_(self.accept[:nb], non_blocking=True)
        if self.draft is not None and self.k > 0:
            self.h_nat[:nb].copy_(self.native[:nb], non_blocking=True)
        if self.ev1 is not None:
            self.ev1.record()
            self.ev1.synchronize()
            self.last_device_ms = self.ev0.elapsed_time(self.ev1)
        self.h2d_bytes = nb * (self.W * 8 + 8 + 8 + self.max_blocks * 4)
        self.d2h_bytes = nb * (self.W * 8 + 4 + (self.k * 8 if self.draft is not None and self.k > 0 else 0))
        self.last_width = W
        return self.h_out[:nb_real].numpy(), self.h_acc[:nb_real].numpy(), self.h_nat[:nb_real].numpy()

    def _capture(self, nb: int, W: Optional[int] = None):
        # Warm-up and capture run on scratch rows only (block 0, state slot 0):
        # a warm-up iteration really executes, and state that is committed
        # rather than rewritten (deferred recurrent commit) must not see it.
        self.win[:nb].zero_()
        self.seq[:nb].zero_()
        self.bt[:nb].zero_()
        self.slots[:nb].zero_()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        W = self.W if W is None else W
        with torch.cuda.stream(s):
            for _ in range(2):
                self._decode_body(nb, W)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._decode_body(nb, W)
        self.graphs[(nb, W)] = g
        # Restore this step's real inputs (still in the pinned staging buffers).
        nbt = self.max_blocks
        self.win[:nb].copy_(self.h_win[:nb], non_blocking=True)
        self.seq[:nb].copy_(self.h_seq[:nb], non_blocking=True)
        self.bt[:nb, :nbt].copy_(self.h_bt[:nb, :nbt], non_blocking=True)
        self.slots[:nb].copy_(self.h_slots[:nb], non_blocking=True)
        return g

    # ------------------------------------------------------------------ prefill
    def prefill(self, prompts: List[np.ndarray], block_tables: List[List[int]],
                state_slots: Optional[List[int]] = None, hidden_only: bool = False, features: bool = False,
                starts: Optional[List[int]] = None, follow: Optional[List[Optional[int]]] = None,
                drafts: bool = True):
        """Prefill a batch of prompts. Returns (first tokens [n], native drafts [n, k]); with
        hidden_only the final normalised hidden state at each prompt's last position [n, H] (scoring);
        with features the target's pre-norm hidden state at every prompt position [sum(len), H] (the draft
        head's input features, for its training replay).

        Chunked prefill: prompts[i] may be the chunk of a longer prompt whose first starts[i] tokens are
        already in the cache (attention-only models); follow[i] is then the prompt token after the chunk
        (the draft head's input at the chunk's last position), or None for a chunk that ends the prompt.
        drafts=False skips the native draft steps (a chunk that does not end its prompt)."""
        dev = self.device
        n = len(prompts)
        lens = [len(p) for p in prompts]
        starts = [0] * n if starts is None else [int(s) for s in starts]
        if self.recurrent and any(starts):
            raise ValueError("chunked prefill needs an attention-only model (recurrent states prefill whole)")
        ids = torch.from_numpy(np.concatenate(prompts).astype(np.int64)).to(dev, non_blocking=True)
        pos = torch.from_numpy(np.concatenate([np.arange(s, s + l) for s, l in zip(starts, lens)]).astype(np.int64)).to(dev)
        mb = max(len(b) for b in block_tables)
        btn = np.zeros((n, mb), dtype=np.int32)
        for i, b in enumerate(block_tables):
            btn[i, :len(b)] = b
        bt = torch.from_numpy(btn).to(dev)
        req_of_tok = torch.from_numpy(np.concatenate([np.full(l, i) for i, l in enumerate(lens)])).to(dev)
        blk = bt.long()[req_of_tok, torch.div(pos, self.bs, rounding_mode="floor")]
        slots = blk * self.bs + pos % self.bs
        seq_lens = torch.tensor([s + l for s, l in zip(starts, lens)], dtype=torch.long, device=dev)
        qs = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.long, device=dev)
        tr, t0 = ops.plan_attention_tiles(lens, self.group)
        meta = AttnMeta(positions=pos, slot_mapping=slots, block_tables=bt, seq_lens=seq_lens, q_start=qs,
                        tile_req=torch.tensor(tr, dtype=torch.int32, device=dev),
                        tile_row0=torch.tensor(t0, dtype=torch.int32, device=dev), num_tokens=int(sum(lens)),
                        nsplit=ops.attention_splits(len(tr), self.model.kv_heads_local, mb),
                        max_rows=_max_rows(max(lens) * self.group))
        slot_t = torch.tensor(state_slots if state_slots is not None else [0] * n, dtype=torch.long, device=dev)
        meta.state_slots, meta.pending, meta.window = slot_t, self.pending, 0
        hid, pre = self.model.forward(ids, meta, self.caches)
        if self.recurrent:
            self.pending.index_fill_(0, slot_t, 0)
        last = qs[1:] - 1
        if features:
            return pre
        if hidden_only:
            return hid.index_select(0, last)
        first = self.model.greedy(hid.index_select(0, last))
        natives = torch.zeros(n, max(self.k, 1), dtype=torch.long, device=dev)
        if self.draft is not None and self.k > 0:
            nxt = torch.empty_like(ids)
            nxt[:-1] = ids[1:]
            nxt[last] = first  # the token after each prompt's last position
            if follow is not None and any(f is not None for f in follow):
                ends = qs[1:].cpu().numpy() - 1
                for i, f in enumerate(follow):
                    if f is not None:
                        nxt[int(ends[i])] = int(f)
            dh, dpre = self.draft.forward(nxt, pre, meta, self.dcaches)
            if drafts:
                d1 = self.model.greedy(dh.index_select(0, last))
                f1 = dpre.index_select(0, last)
                natives = self._draft_steps(d1, f1, seq_lens, bt, n)
        return first.cpu().numpy(), natives.cpu().numpy()
