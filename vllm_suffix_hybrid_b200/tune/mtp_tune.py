"""Online, idle-time fine-tuning of the draft head (SUFFIX_MTP_TUNE=1, default off).

Drafts are always verified by the target, so a better-matched draft head only changes speed.  This
trains zero-initialised low-rank adapters on the draft head's dense linears from the traffic the
engine serves, between requests, and promotes them only when a paired replay on held-out requests shows
a longer mean accepted length.  Reference behaviour: suffix_hybrid/mtp_tune/__init__.py:1-80 (capture
sample, adapters, teacher-forced training, gated promotion, idle scheduling, shadow / rollback, env).

  capture   finished requests whose crc32(request id) falls in the SUFFIX_MTP_TUNE_RATE share keep their
            token sequence (prompt + output); SUFFIX_MTP_TUNE_HELDOUT_PCT of them are held out for the
            gate.  FIFO eviction by a token budget (SUFFIX_MTP_TUNE_MEM_TOKENS).  Only tokens are kept:
            the target's hidden states are recomputed by a target forward at training time, so serving
            pays nothing (the reference copies hidden rows off the serving path instead).
  adapters  A [r, in] (small random) and B [out, r] (zero) per linear (Linear.lora), sharded like the
            weight under tensor parallelism (column: B sharded, row: A sharded), so serving needs no
            extra collective; the live tensors are only updated in place (captured graphs see them).
  training  depth-1 teacher-forced cross-entropy of the head replayed differentiably (tune/replay.py),
            AdamW on fp32 masters of a candidate adapter set, SUFFIX_MTP_TUNE_ACCUM sequences per step,
            each idle micro-step bounded by SUFFIX_MTP_TUNE_STEP_MS.
  gate      every SUFFIX_MTP_TUNE_EVAL_EVERY optimizer steps: greedy draft chains (depth 1..k) replayed
            from every position of the held-out sequences with the live and the candidate adapters;
            promote when the candidate's mean accepted length is higher by SUFFIX_MTP_TUNE_MARGIN over at
            least SUFFIX_MTP_TUNE_MIN_ANCHORS anchors (SUFFIX_MTP_TUNE_SHADOW=1: never promote).
  control   micro-steps run only while the engine has no work (after SUFFIX_MTP_TUNE_IDLE_GRACE_MS);
            touching SUFFIX_MTP_TUNE_ROLLBACK_FILE zeroes the live adapters (an exact no-op) and stops
            promotions; any exception disables tuning, rank-uniformly (a liveness all-reduce).
"""
from __future__ import annotations

import logging
import math
import os
import time
import zlib
from collections import deque
from typing import Dict, Optional

import numpy as np
import torch

from . import replay
from .collectives import allreduce_grads

logger = logging.getLogger(__name__)


def _env(name: str, default, cast=float):
    raw = os.environ.get("SUFFIX_MTP_TUNE_" + name, "").strip()
    return cast(raw) if raw else default


class TuneConfig:
    def __init__(self):
        self.rate = _env("RATE", 0.25)
        self.heldout_pct = _env("HELDOUT_PCT", 20, int)
        self.rank = _env("RANK", 16, int)
        self.alpha = _env("ALPHA", 32.0)
        self.targets = tuple(t for t in _env("TARGETS", ",".join(replay.TARGETS), str).split(",") if t)
        self.lr = _env("LR", 1e-4)
        self.accum = _env("ACCUM", 4, int)
        self.step_ms = _env("STEP_MS", 50.0)
        self.eval_every = _env("EVAL_EVERY", 50, int)
        self.eval_windows = _env("EVAL_WINDOWS", 64, int)
        self.min_eval_windows = _env("MIN_EVAL_WINDOWS", 8, int)
        self.min_train_windows = _env("MIN_TRAIN_WINDOWS", 8, int)
        self.margin = _env("MARGIN", 0.05)
        self.min_anchors = _env("MIN_ANCHORS", 2000, int)
        self.max_len = _env("MAX_LEN", 1024, int)
        self.mem_tokens = _env("MEM_TOKENS", 4_000_000, int)
        self.idle_grace_ms = _env("IDLE_GRACE_MS", 200.0)
        self.shadow = _env("SHADOW", "0", str) == "1"
        self.rollback_file = _env("ROLLBACK_FILE", "/tmp/suffix_mtp_tune.rollback", str)
        self.log_s = _env("LOG_S", 60.0)


def supported(draft) -> bool:
    L = getattr(draft, "layer", None)
    return (L is not None and hasattr(L, "attn") and hasattr(getattr(L, "attn", None), "qkv")
            and hasattr(L, "mlp") and hasattr(draft, "fc") and hasattr(draft, "target"))


class MtpTuner:
    def __init__(self, engine, cfg: Optional[TuneConfig] = None):
        self.engine = engine
        self.draft = engine.draft
        self.cfg = cfg or TuneConfig()
        self.k = max(engine.k, 1)
        self.lin = {n: l for n, l in replay.linears(self.draft).items() if n in self.cfg.targets}
        self.scale = self.cfg.alpha / self.cfg.rank
        g = torch.Generator(device="cpu").manual_seed(1234)  # identical on every rank
        self.live: Dict[str, tuple] = {}
        self.cand: Dict[str, tuple] = {}
        params = []
        for n, lin in self.lin.items():
            out_f, in_f = lin.weight.shape
            a0 = torch.randn(self.cfg.rank, in_f, generator=g) / math.sqrt(in_f)
            a = a0.to(lin.weight.device, lin.weight.dtype, copy=True)  # live and candidate never share storage
            b = torch.zeros(out_f, self.cfg.rank, device=lin.weight.device, dtype=lin.weight.dtype)
            lin.lora = (a, b, self.scale)
            lin.push = False  # the adapter adds to the materialised partial output
            self.live[n] = (a, b)
            ca = torch.nn.Parameter(a0.to(lin.weight.device, torch.float32, copy=True))
            cb = torch.nn.Parameter(torch.zeros(out_f, self.cfg.rank, device=lin.weight.device))
            self.cand[n] = (ca, cb)
            params += [ca, cb]
        self.params = params
        self.opt = torch.optim.AdamW(params, lr=self.cfg.lr, weight_decay=0.0)
        self.train: deque = deque()
        self.heldout: deque = deque()
        self.tokens_kept = 0
        self._cursor = 0
        self._accum = 0
        self.disabled = False
        self.promote_ok = True
        self.last_work = time.monotonic()
        self.stats = {"captured": 0, "heldout": 0, "opt_steps": 0, "micro_steps": 0, "evals": 0, "promotions": 0,
                      "last_live_accept": 0.0, "last_cand_accept": 0.0, "last_loss": 0.0, "reason": ""}
        self._last_log = time.monotonic()

    @classmethod
    def from_env(cls, engine) -> Optional["MtpTuner"]:
        if os.environ.get("SUFFIX_MTP_TUNE", "").strip() != "1":
            return None
        if engine.draft is None or engine.k == 0:
            logger.warning("SUFFIX_MTP_TUNE: no draft head to tune")
            return None
        if not supported(engine.draft):
            logger.warning("SUFFIX_MTP_TUNE: draft head %s has no training replay: tuning off",
                           type(engine.draft).__name__)
            return None
        return cls(engine)

    # ------------------------------------------------------------------ capture
    def capture(self, rid: str, seq: np.ndarray) -> None:
        h = zlib.crc32(rid.encode())
        if h >= self.cfg.rate * 2 ** 32 or len(seq) < 4:
            return
        seq = np.asarray(seq[: self.cfg.max_len], dtype=np.int64)
        dst = self.heldout if (h % 100) < self.cfg.heldout_pct else self.train
        dst.append(seq)
        self.tokens_kept += len(seq)
        self.stats["captured"] += 1
        self.stats["heldout"] = len(self.heldout)
        while self.tokens_kept > self.cfg.mem_tokens and (self.train or self.heldout):
            src = self.train if len(self.train) >= len(self.heldout) else self.heldout
            self.tokens_kept -= len(src.popleft())

    def note_work(self) -> None:
        self.last_work = time.monotonic()

    def wants_step(self) -> bool:
        return (not self.disabled and len(self.train) >= self.cfg.min_train_windows
                and (time.monotonic() - self.last_work) * 1e3 >= self.cfg.idle_grace_ms)

    # ------------------------------------------------------------------ training
    def _ad(self, which: str) -> dict:
        src = self.live if which == "live" else self.cand
        return {n: (a, b, self.scale) for n, (a, b) in src.items()}

    def _feats(self, seq: np.ndarray) -> torch.Tensor:
        return self.engine.features(seq).float()

    def micro_step(self) -> bool:
        """One bounded slice of training / gating between requests; False when nothing ran."""
        if self.disabled:
            return False
        ok = True
        ran = False
        try:
            if os.path.exists(self.cfg.rollback_file):
                self.rollback()
                return False
            if len(self.train) < self.cfg.min_train_windows:
                return False
            t0 = time.perf_counter()
            while (time.perf_counter() - t0) * 1e3 < self.cfg.step_ms:
                seq = self.train[self._cursor % len(self.train)]
                self._cursor += 1
                st = torch.from_numpy(seq).to(self.draft.fc.device)
                with torch.enable_grad():
                    loss, n = replay.train_loss(self.draft, self._ad("cand"), st, self._feats(seq))
                    if loss is None:
                        continue
                    (loss / self.cfg.accum).backward()
                self.stats["last_loss"] = float(loss.detach())
                ran = True
                self._accum += 1
                if self._accum >= self.cfg.accum:
                    self._opt_step()
            self.stats["micro_steps"] += int(ran)
        except Exception as exc:
            ok = False
            self.stats["reason"] = f"{type(exc).__name__}: {exc}"
            logger.exception("[mtp-tune] disabled after an exception")
        if not self._vote(ok):
            self.disabled = True
        self._log()
        return ran

    def _opt_step(self) -> None:
        allreduce_grads(self._replicated_params())
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        self._accum = 0
        self.stats["opt_steps"] += 1
        if self.stats["opt_steps"] % self.cfg.eval_every == 0:
            self.evaluate()

    def _replicated_params(self):
        """Adapter factors that every TP rank holds whole (their gradients are summed over ranks)."""
        out = []
        for n, (a, b) in self.cand.items():
            par = self.lin[n].parallel
            if par == "col":
                out.append(a)
            elif par == "row":
                out.append(b)
        return out

    # ------------------------------------------------------------------ gate
    @torch.no_grad()
    def evaluate(self) -> Optional[tuple]:
        seqs = list(self.heldout)[-self.cfg.eval_windows:]
        if len(seqs) < self.cfg.min_eval_windows:
            return None
        live_sum = cand_sum = 0.0
        anchors_n = 0
        for seq in seqs:
            st = torch.from_numpy(seq).to(self.draft.fc.device)
            feats = self._feats(seq)
            anchors = torch.arange(0, len(seq) - 2, device=st.device)
            if anchors.numel() == 0:
                continue
            live_sum += float(replay.chain_accept(self.draft, self._ad("live"), st, feats, anchors, self.k).sum())
            cand_sum += float(replay.chain_accept(self.draft, self._ad("cand"), st, feats, anchors, self.k).sum())
            anchors_n += anchors.numel()
        self.stats["evals"] += 1
        if anchors_n == 0:
            return None
        live, cand = 1.0 + live_sum / anchors_n, 1.0 + cand_sum / anchors_n  # tokens per step incl. bonus
        self.stats["last_live_accept"], self.stats["last_cand_accept"] = live, cand
        promote = (anchors_n >= self.cfg.min_anchors and cand - live >= self.cfg.margin and not self.cfg.shadow
                   and self.promote_ok)
        if promote:
            self.promote()
        logger.warning("[mtp-tune] gate anchors=%d live=%.4f candidate=%.4f -> %s", anchors_n, live, cand,
                       "promote" if promote else "keep")
        return live, cand, anchors_n, promote

    @torch.no_grad()
    def promote(self) -> None:
        """Candidate -> live adapters, in place (between engine steps)."""
        for n, (a, b) in self.live.items():
            ca, cb = self.cand[n]
            a.copy_(ca.to(a.dtype))
            b.copy_(cb.to(b.dtype))
        self.stats["promotions"] += 1

    @torch.no_grad()
    def rollback(self) -> None:
        for _, b in self.live.values():
            b.zero_()  # B = 0: the adapter adds exactly zero
        self.promote_ok = False
        self.stats["reason"] = "rolled back"

    # ------------------------------------------------------------------ rank agreement / telemetry
    def _vote(self, ok: bool) -> bool:
        from ..parallel import state

        st = state.get()
        if st.tp <= 1:
            return ok
        import torch.distributed as dist

        t = torch.tensor([1 if ok else 0], dtype=torch.int32)
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=st.cpu_group)
        return bool(t.item())

    def _log(self) -> None:
        if time.monotonic() - self._last_log >= self.cfg.log_s:
            self._last_log = time.monotonic()
            logger.warning("[mtp-tune] %s", self.stats)
