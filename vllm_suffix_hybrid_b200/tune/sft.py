"""In-place supervised fine-tuning of the served model (SUFFIX_SFT=1, default off).

There is one model: zero-initialised low-rank adapters are attached to the served model's linears at
load time (Linear.lora, before any graph capture), so every request already runs base + adapter.  A
training run replays the same weights differentiably (tune/replay.py target_logits, per-layer
recomputation), keeps fp32 master copies and AdamW state of the adapters in host memory (only the
working adapters and their gradients live on the GPU), runs one optimizer step per engine-loop slice
between serving steps, and at the end copies the trained values into the live adapter tensors in
place: the next serving step uses them.  Runs are checkpointed per rank under SUFFIX_SFT_DIR
(runs/<id>/adapter-tp<r>-of-<n>.safetensors, metadata.json) with an atomically replaced latest.json
that the next start restores.  Reference behaviour: suffix_hybrid/sft/__init__.py:1-70 and
sft/api.py:1-40 (routes, final-assistant-turn loss, latest.json restore, fail-closed restore).

Deviations: Llama-family targets only (other architectures log a reason and stay off), checkpoints
are local (no Hub upload: no network), no served-vs-trained parity gate (the replay is tested equal
to the serving forward instead).
Env: SUFFIX_SFT_RANK=16 / _ALPHA=32 / _TARGETS=glob,... (names like layers.3.qkv) / _DIR / _MAX_EXAMPLES=256
/ _MAX_STEPS=1000 / _MAX_TOKENS=4096 / _DUTY=0.5 (training share of engine-loop time under load).
"""
from __future__ import annotations

import fnmatch
import json
import logging
import math
import os
import time
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

from ..parallel import state
from . import replay
from .collectives import allreduce_grads

logger = logging.getLogger(__name__)


def _env(name, default, cast=str):
    raw = os.environ.get("SUFFIX_SFT_" + name, "").strip()
    return cast(raw) if raw else default


def supported(model) -> Optional[str]:
    """None when the model can be trained in place, else the reason."""
    layers = getattr(model, "layers", None)
    if not layers:
        return "no decoder layers"
    for L in layers:
        if not (hasattr(L, "attn") and hasattr(L.attn, "qkv") and hasattr(L, "mlp") and hasattr(L.mlp, "gate_up")):
            return f"layer type {type(L).__name__} has no training replay (MLA / GDN / MoE layers are refused)"
    return None


class SftTrainer:
    def __init__(self, engine):
        self.engine = engine
        self.model = engine.model
        self.rank = _env("RANK", 16, int)
        self.scale = _env("ALPHA", 32.0, float) / self.rank
        pats = [p for p in _env("TARGETS", "*", str).split(",") if p]
        self.lin = {n: l for n, l in replay.target_linears(self.model).items()
                    if any(fnmatch.fnmatch(n, p) for p in pats)}
        self.dir = _env("DIR", os.path.join(os.path.expanduser("~"), ".cache", "suffix_sft"), str)
        self.max_examples = _env("MAX_EXAMPLES", 256, int)
        self.max_steps = _env("MAX_STEPS", 1000, int)
        self.max_tokens = _env("MAX_TOKENS", 4096, int)
        self.duty = _env("DUTY", 0.5, float)
        g = torch.Generator(device="cpu").manual_seed(4321)  # identical on every rank
        self.live: Dict[str, tuple] = {}
        self.master: Dict[str, List[torch.Tensor]] = {}
        self.work: Dict[str, List[torch.Tensor]] = {}
        for n, lin in self.lin.items():
            out_f, in_f = lin.weight.shape
            a0 = torch.randn(self.rank, in_f, generator=g) / math.sqrt(in_f)
            a = a0.to(lin.weight.device, lin.weight.dtype, copy=True)
            b = torch.zeros(out_f, self.rank, device=lin.weight.device, dtype=lin.weight.dtype)
            lin.lora = (a, b, self.scale)
            lin.push = False
            self.live[n] = (a, b)
            self.master[n] = [a0.clone(), torch.zeros(out_f, self.rank)]
        self.run: Optional[dict] = None
        self.status = {"state": "idle", "run_id": "base", "step": 0, "steps": 0, "loss": None, "error": ""}
        self._train_s = 0.0
        self._t0 = time.monotonic()

    @classmethod
    def from_env(cls, engine) -> Optional["SftTrainer"]:
        if os.environ.get("SUFFIX_SFT", "").strip() != "1":
            return None
        why = supported(engine.model)
        if why is not None:
            logger.warning("SUFFIX_SFT off: %s", why)
            return None
        t = cls(engine)
        t.restore()
        return t

    # ------------------------------------------------------------------ runs
    def begin(self, examples: List[Tuple[List[int], List[int]]], steps: int = 1, batch_size: int = 1,
              learning_rate: float = 1e-4, weight_decay: float = 0.0, run_id: Optional[str] = None) -> str:
        if self.status["state"] == "restore_failed":
            raise RuntimeError("a checkpoint restore failed: load a run (or base) before training")
        if self.run is not None:
            raise RuntimeError("a training run is in progress")
        if not examples or len(examples) > self.max_examples:
            raise ValueError(f"1 to {self.max_examples} examples required")
        if not 1 <= steps <= self.max_steps:
            raise ValueError(f"steps must be 1..{self.max_steps}")
        for p, t in examples:
            if not t or len(p) + len(t) > self.max_tokens:
                raise ValueError(f"every example needs target tokens and at most {self.max_tokens} tokens")
        dev = next(iter(self.live.values()))[0].device
        self.work = {n: [m.to(dev, torch.float32, copy=True).requires_grad_(True) for m in ms]
                     for n, ms in self.master.items()}
        params = [m for ms in self.master.values() for m in ms]
        for m in params:
            m.grad = None
        self.run = {"examples": examples, "steps": steps, "batch": max(1, batch_size), "cursor": 0,
                    "opt": torch.optim.AdamW(params, lr=learning_rate, weight_decay=weight_decay),
                    "run_id": run_id or time.strftime("%Y%m%d-%H%M%S")}
        self.status.update(state="training", step=0, steps=steps, loss=None, error="", run=self.run["run_id"])
        return self.run["run_id"]

    def _loss(self, prompt: List[int], target: List[int]) -> torch.Tensor:
        dev = next(iter(self.work.values()))[0].device
        toks = torch.tensor(list(prompt) + list(target), dtype=torch.long, device=dev)
        ad = {n: (w[0], w[1], self.scale) for n, w in self.work.items()}
        logits = replay.target_logits(self.model, ad, toks[:-1])
        p = len(prompt)
        return F.cross_entropy(logits[p - 1:], toks[p:])  # loss on the target tokens only

    def wants_step(self, busy: bool) -> bool:
        if self.run is None:
            return False
        if not busy:
            return True
        return self._train_s <= self.duty * max(time.monotonic() - self._t0, 1e-3)

    def micro(self) -> bool:
        """One optimizer step of the active run (then commit + save when it is the last); False when idle."""
        r = self.run
        if r is None:
            return False
        t0 = time.monotonic()
        try:
            ex = r["examples"]
            total = 0.0
            for _ in range(r["batch"]):
                p, t = ex[r["cursor"] % len(ex)]
                r["cursor"] += 1
                with torch.enable_grad():
                    loss = self._loss(p, t) / r["batch"]
                    loss.backward()
                total += float(loss.detach())
            allreduce_grads(self._replicated())
            for n, ws in self.work.items():  # gradients to the host masters, AdamW on the host
                for w, m in zip(ws, self.master[n]):
                    m.grad = w.grad.detach().cpu() if w.grad is not None else torch.zeros_like(m)
                    w.grad = None
            r["opt"].step()
            r["opt"].zero_grad(set_to_none=True)
            with torch.no_grad():
                for n, ws in self.work.items():
                    for w, m in zip(ws, self.master[n]):
                        w.copy_(m.to(w.device))
            self.status["step"] += 1
            self.status["loss"] = total
            if self.status["step"] >= r["steps"]:
                self.commit()
                self.save(r["run_id"])
                self.run = None
                self.status.update(state="idle", run_id=r["run_id"])
        except Exception as exc:
            logger.exception("SFT run failed")
            self.run = None
            self.status.update(state="failed", error=f"{type(exc).__name__}: {exc}")
        self._train_s += time.monotonic() - t0
        return True

    def _replicated(self):
        out = []
        for n, (a, b) in self.work.items():
            par = self.lin[n].parallel
            if par == "col":
                out.append(a)
            elif par == "row":
                out.append(b)
        return out

    @torch.no_grad()
    def commit(self) -> None:
        """Masters -> live adapters, in place (between serving steps)."""
        for n, (a, b) in self.live.items():
            a.copy_(self.master[n][0].to(a.device, a.dtype))
            b.copy_(self.master[n][1].to(b.device, b.dtype))

    # ------------------------------------------------------------------ checkpoints
    def _shard_name(self) -> str:
        st = state.get()
        return f"adapter-tp{st.tp_rank}-of-{st.tp}.safetensors"

    def save(self, run_id: str) -> str:
        from safetensors.torch import save_file

        d = os.path.join(self.dir, "runs", run_id)
        os.makedirs(d, exist_ok=True)
        tensors = {}
        for n, (a, b) in self.master.items():
            tensors[n + ".A"] = a.contiguous()
            tensors[n + ".B"] = b.contiguous()
        save_file(tensors, os.path.join(d, self._shard_name()))
        if state.get().rank == 0:
            meta = {"run_id": run_id, "rank": self.rank, "alpha": self.scale * self.rank,
                    "targets": sorted(self.master), "tp": state.get().tp, "time": time.time()}
            with open(os.path.join(d, "metadata.json"), "w") as fh:
                json.dump(meta, fh)
            self._set_latest(run_id)
        return d

    def _set_latest(self, run_id: str) -> None:
        os.makedirs(self.dir, exist_ok=True)
        tmp = os.path.join(self.dir, "latest.json.tmp")
        with open(tmp, "w") as fh:
            json.dump({"run_id": run_id}, fh)
        os.replace(tmp, os.path.join(self.dir, "latest.json"))

    def load(self, run_id: str) -> None:
        """Serve a saved run ("base" = zero adapters) and make it the one restored at the next start."""
        if self.run is not None:
            raise RuntimeError("a training run is in progress")
        if run_id == "base":
            for n in self.master:
                self.master[n][1].zero_()
        else:
            from safetensors.torch import load_file

            path = os.path.join(self.dir, "runs", run_id, self._shard_name())
            if not os.path.exists(path):
                raise FileNotFoundError(f"no checkpoint for run {run_id!r} on this rank")
            t = load_file(path)
            if sorted(k[:-2] for k in t if k.endswith(".A")) != sorted(self.master):
                raise ValueError("checkpoint adapters do not match this model's targets")
            for n in self.master:
                if t[n + ".A"].shape != self.master[n][0].shape or t[n + ".B"].shape != self.master[n][1].shape:
                    raise ValueError(f"adapter {n} shape differs (rank / tensor-parallel layout)")
                self.master[n][0].copy_(t[n + ".A"])
                self.master[n][1].copy_(t[n + ".B"])
        self.commit()
        if state.get().rank == 0:
            self._set_latest(run_id)
        self.status.update(state="idle", run_id=run_id, error="")

    def restore(self) -> None:
        """Load the run latest.json names (if any); a failure keeps the base model and refuses training."""
        path = os.path.join(self.dir, "latest.json")
        if not os.path.exists(path):
            return
        try:
            with open(path) as fh:
                run_id = json.load(fh)["run_id"]
            self.load(run_id)
        except Exception as exc:
            logger.warning("SFT restore failed (%s): serving the base model", exc)
            self.status.update(state="restore_failed", error=f"{type(exc).__name__}: {exc}")
