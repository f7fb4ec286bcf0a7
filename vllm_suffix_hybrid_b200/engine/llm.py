"""Public engine API: add requests, step, generate.

A step either prefills newly admitted requests (batched up to
``max_prefill_tokens`` prompt tokens), prefills the next ``max_prefill_tokens``
chunk of one longer prompt (such chunks alternate with decode steps, so a long
prompt does not stall the running requests), or runs one speculative decode
step for every running request.  After each step the proposer picks the next
drafts:

* ``hybrid``  -- native drafts (EAGLE/MTP head) mixed with the suffix corpus
  by the native HybridMixer (legacy split or diverge), fed the verified
  accepted lengths;
* ``native``  -- native drafts only;
* ``suffix``  -- drafter-free V2SuffixProposer (uniform-k pallet);
* ``ngram``   -- weight-free Engine (suffix corpus + in-request n-gram);
* ``external``-- drafts from a user callable ``engine.external_proposer(requests)
  -> list[list[int]]`` (a custom drafter hook);
* ``none``    -- plain one-token decode.

Running requests occupy rows 0..B-1 of the host token buffer in batch order
(a finished request's row is back-filled by the last one), so the proposers
read every context in place.
"""
from __future__ import annotations

import itertools
import logging
import os
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from .. import _native
from ..models import build_model
from ..parallel import state as pstate
from .config import EngineConfig, apply_env
from .kv_cache import BlockPool, allocate_caches, blocks_for
from .runner import Runner
from .telemetry import Telemetry

logger = logging.getLogger(__name__)


def _trace_budget(name: str) -> list:
    """[remaining traced steps] of SUFFIX_HYBRID_<name> (0 = off; _MAX sets the budget, default 24)."""
    import os

    if not os.environ.get("SUFFIX_HYBRID_" + name, "").strip():
        return [0]
    try:
        return [max(0, int(os.environ.get("SUFFIX_HYBRID_" + name + "_MAX", "") or 24))]
    except ValueError:
        return [24]


@dataclass
class Request:
    rid: str
    prompt: np.ndarray
    max_new_tokens: int
    output: List[int] = field(default_factory=list)
    blocks: List[int] = field(default_factory=list)
    blocks_np: np.ndarray = field(default_factory=lambda: np.zeros(0, dtype=np.int32))  # int32 mirror of blocks
    committed: int = 0  # KV positions written and verified
    next_token: int = -1  # bonus token waiting for the next window
    drafts: List[int] = field(default_factory=list)
    accepted_prev: int = -1  # accepted length of the previous proposal (-1 = none)
    finished: bool = False
    arrival: float = 0.0
    slot: int = 0  # recurrent-state slot (hybrid GDN models)
    stop_ids: frozenset = frozenset()  # generation ends after the first of these tokens
    finish_reason: str = ""  # "length" | "stop" | "abort"
    polled: int = 0  # output tokens already handed out by poll()
    prefilled: int = 0  # prompt tokens in the cache while a long prompt is prefilled in chunks

    @property
    def history_len(self) -> int:
        return len(self.prompt) + len(self.output)


@dataclass
class StepStats:
    kind: str
    num_reqs: int
    emitted: int
    accepted: int
    device_ms: float
    host_ms: float
    proposer_us: float


class LLMEngine:
    def __init__(self, cfg: EngineConfig):
        self.cfg = apply_env(cfg)
        st = pstate.get()
        dev = cfg.device
        if torch.device(dev).type == "cuda":
            dev = f"cuda:{st.local_rank}" if ":" not in dev else dev
            torch.cuda.set_device(torch.device(dev))
        self.device = dev
        torch.manual_seed(cfg.seed)
        mcfg = cfg.model
        spec = cfg.spec
        self.k = spec.k if spec.method != "none" else 0
        self.adaptive_width = bool(getattr(spec, "adaptive_width", True))
        # The RoPE tables are indexed by position on the device: they must cover every position a request of
        # max_model_len can write (its prompt, its output and the verify look-ahead), or a decode step reads
        # past the table.  Rotary embeddings are defined for any position, so the table is extended.
        reach = cfg.cache.max_model_len + 2 * self.k + 2
        if mcfg.max_position < reach:
            logger.warning("RoPE table extended from %d to %d positions (max_model_len %d)", mcfg.max_position,
                           reach, cfg.cache.max_model_len)
            mcfg.max_position = reach
        self.model, self.draft = build_model(mcfg, dev, cfg.seed, with_draft=spec.method in ("hybrid", "native"))
        if (st.tp > 1 or st.ep > 1) and cfg.parallel.comm == "fused" and torch.device(dev).type == "cuda":
            from ..parallel import comm as pcomm
            from ..parallel.symm import SymmComm

            max_tok = max(cfg.max_prefill_tokens, cfg.max_num_seqs * (spec.k + 1))
            pcomm.set_fused(SymmComm(mcfg.hidden, max_tok))
        if cfg.weights:
            from .loader import load_weights

            load_weights(self.model, self.draft, cfg.weights)
        from ..models import lm_head

        if lm_head.enabled() and lm_head.install(self.model) is not None:
            logger.warning("NVFP4-screened LM head active (max M %d, re-score %d)", self.model.lm_screen.max_m,
                           self.model.lm_screen.rescore)
        bs = cfg.cache.block_size
        self.block_size = bs
        self.max_model_len = cfg.cache.max_model_len
        self.max_blocks_per_seq = blocks_for(self.max_model_len + 2 * self.k + 2, bs)
        self.host_tier = None
        if cfg.cache.host_kv:
            from .host_tier import hot_rows_for

            if not hasattr(self.model, "enable_host_kv"):
                raise ValueError("the host KV tier needs a DSA sparse-attention model (DeepSeek-V3.2 shape)")
            self.model.enable_host_kv(cfg.cache.host_kv_hot_rows or hot_rows_for(self.k, mcfg.dsa_topk),
                                      self.max_model_len + 2 * self.k + 2, cfg.max_num_seqs * (self.k + 1))
        num_blocks = cfg.cache.num_blocks or self._auto_blocks()
        self.pool = BlockPool(num_blocks)
        if hasattr(self.model, "allocate_caches"):
            self.caches = self.model.allocate_caches(num_blocks, bs, cfg.max_num_seqs + 1, self.k + 1)
            self.host_tier = getattr(self.model, "host_tier", None)
        else:
            self.caches = allocate_caches(mcfg.layers, self.model.kv_cache_shape(num_blocks, bs), self.model.dtype,
                                          dev)
        if self.draft is None:
            self.dcaches = None
        elif hasattr(self.draft, "allocate_caches"):
            self.dcaches = self.draft.allocate_caches(num_blocks, bs)
        else:
            self.dcaches = allocate_caches(1, self.model.kv_cache_shape(num_blocks, bs), self.model.dtype, dev)[0]
        self._free_slots = list(range(cfg.max_num_seqs, 0, -1))
        self.runner = Runner(self.model, self.draft, self.caches, self.dcaches, self.k, cfg.max_num_seqs,
                             self.max_blocks_per_seq, bs, dev, cfg.cuda_graphs)
        self.tokens = np.zeros((cfg.max_num_seqs, self.max_model_len + 2 * self.k + 2), dtype=np.int64)
        self.running: List[Request] = []
        self.waiting: List[Request] = []
        self.prefilling: Optional[Request] = None  # a long prompt being prefilled in chunks
        self._last_kind = ""  # "chunk" after a chunked-prefill step, "decode" after a decode step
        self.finished: Dict[str, Request] = {}
        self._ids = itertools.count()
        self.stats: List[StepStats] = []
        self.proposer = None
        self.telemetry = Telemetry.from_env()
        from ..utils.step_profiler import StepProfiler

        self.step_profiler = StepProfiler.from_env(st.rank)
        self.external_proposer = None  # callable(list[Request]) -> list[list[int]] for method "external"
        k = max(self.k, 1)
        if spec.method == "hybrid":
            self.proposer = _native.HybridMixer(k, self.tokens.shape[1])
        elif spec.method == "suffix":
            self.proposer = _native.V2SuffixProposer(k, self.tokens.shape[1], spec.min_len, spec.uniform_k,
                                                    spec.width_gate)
        elif spec.method == "ngram":
            self.proposer = _native.Engine(k, self.tokens.shape[1])
        # Async scheduling (lag-1 drafting, SUFFIX_HYBRID_ASYNC=1): suffix / hybrid only; other methods keep
        # synchronous scheduling (the reference's sched_sync rule, sched_sync.py:85).
        self._pipe = None
        self.dp = st.dp
        self._async = bool(spec.async_scheduling and self.k > 0 and spec.method in ("suffix", "hybrid")
                           and self.dp == 1)
        if spec.async_scheduling and not self._async:
            logger.warning("SUFFIX_HYBRID_ASYNC ignored for method %r: synchronous scheduling", spec.method)
        self._cand_len = 2 * self.k + 1
        self.async_proposer = (_native.V2SuffixProposer(self._cand_len, self.tokens.shape[1], spec.min_len, False,
                                                        False) if self._async else None)
        self._hyb_min = (spec.async_hyb_min or self.k) if spec.method == "hybrid" else 0
        self._lag = self.k + 1 if self._async else 0  # tokens a lagged step may add beyond the host's view
        self._trace_verify = _trace_budget("TRACE_VERIFY2")
        self._trace_sched = _trace_budget("SCHEDTRACE")
        from ..tune.mtp_tune import MtpTuner

        self.tuner = MtpTuner.from_env(self)  # SUFFIX_MTP_TUNE=1: adapters attach before any graph capture
        # SUFFIX_HYBRID_CORPUS_FILE: the suffix corpus is restored from this snapshot at start (when it exists)
        # and written back by save_corpus() (the HTTP server does so at shutdown)
        self.corpus_file = os.environ.get("SUFFIX_HYBRID_CORPUS_FILE") or None
        if self.corpus_file and os.path.exists(self.corpus_file) and self._corpus_caches():
            n = self.load_corpus(self.corpus_file)
            logger.warning("suffix corpus restored from %s: %d sequences", self.corpus_file, n)
        from ..tune.sft import SftTrainer

        self.sft = SftTrainer.from_env(self)  # SUFFIX_SFT=1: adapters on the served model, before capture

    # ------------------------------------------------------------------ sizing
    def _auto_blocks(self) -> int:
        """KV blocks from the memory budget: at most 4x what max_num_seqs full-length requests could hold,
        at least one full-length request.  Requests are admitted against their own reservations
        (`_select_prefill`), so a pool smaller than max_num_seqs full-length requests never runs dry; it
        only admits fewer long requests at once."""
        c = self.cfg
        need = c.max_num_seqs * (self.max_blocks_per_seq + 1) + 8
        if torch.device(self.device).type != "cuda":
            return need
        free, _ = torch.cuda.mem_get_info()
        m = self.model
        kv_layers = getattr(m, "num_kv_layers", c.model.layers)
        if hasattr(m, "kv_block_bytes"):  # latent-cache models size their own rows (MLA: NVFP4 or bf16 + indexer)
            per_block = m.kv_block_bytes(self.block_size) * kv_layers
            if self.draft is not None:
                per_block += (self.draft.kv_block_bytes(self.block_size) if hasattr(self.draft, "kv_block_bytes")
                              else m.kv_block_bytes(self.block_size))
        else:
            per_block = 2 * self.block_size * m.kv_heads_local * c.model.head_dim * m.embed.element_size()
            per_block *= kv_layers + (1 if self.draft is not None else 0)
        budget = int(free * c.cache.gpu_memory_fraction) - (4 << 30)
        if c.cache.host_kv and hasattr(m, "latent_block_bytes"):  # latent rows in host memory, hot rows on device
            hot = m.host_kv[0] * (c.max_num_seqs + 1) * m.latent_block_bytes(1) * kv_layers
            budget -= hot
            host = int(c.cache.host_kv_gb * (1 << 30)) // (m.latent_block_bytes(self.block_size) * kv_layers)
            return max(self.max_blocks_per_seq + 9, min(budget // max(per_block, 1), host, 4 * need))
        return max(self.max_blocks_per_seq + 9, min(budget // per_block, 4 * need))

    # ------------------------------------------------------------------ API
    def add_request(self, prompt, max_new_tokens: int = 128, rid: Optional[str] = None,
                    stop_token_ids=None) -> str:
        rid = rid if rid is not None else f"req-{next(self._ids)}"
        p = np.asarray(prompt, dtype=np.int64)
        if len(p) == 0 or len(p) + max_new_tokens > self.max_model_len:
            raise ValueError("prompt empty or prompt + max_new_tokens exceeds max_model_len")
        if (rid in self.finished or any(r.rid == rid for r in self.running) or any(r.rid == rid for r in self.waiting)
                or (self.prefilling is not None and self.prefilling.rid == rid)):
            raise ValueError(f"duplicate request id {rid}")
        self.waiting.append(Request(rid, p, max_new_tokens, arrival=time.time(),
                                    stop_ids=frozenset(int(t) for t in (stop_token_ids or ()))))
        return rid

    def admit_prefilled(self, prompts, max_new_tokens: int = 128, seed: int = 0) -> List[str]:
        """Benchmark helper: admit requests as if their prompts had been prefilled, without the prefill pass.

        Decode throughput at long contexts (32k-128k tokens per request) is measured on a cache of the
        right size; a real prefill of millions of prompt tokens would dominate the run.  The requests get
        their blocks, slot and token history (the proposers see the full prompt), the cache contents are
        set once to random values of the cache's format (finite bf16 / fp8 / NVFP4 codes; recurrent
        states zero), and each request's first output token is drawn at random.  Every decode step after
        this does its full work; only the prefill forward is skipped.
        """
        rng = np.random.default_rng(seed)
        if not getattr(self, "_synthetic_cache", False):
            self._fill_caches_random(seed)
            self._synthetic_cache = True
        rids = []
        for p in prompts:
            if len(self.running) + (self.prefilling is not None) >= self.cfg.max_num_seqs:
                raise RuntimeError("admit_prefilled: more requests than max_num_seqs")
            rid = self.add_request(p, max_new_tokens)
            r = self.waiting.pop()
            if self._reservation(r) > self._unclaimed_blocks():
                raise MemoryError(f"admit_prefilled: request {rid} does not fit the KV blocks left unpromised")
            self._ensure_blocks(r, len(r.prompt) + 2 * self.k + 2)
            r.slot = self._free_slots.pop()
            row = len(self.running)
            self.running.append(r)
            self.tokens[row, :len(r.prompt)] = r.prompt
            r.committed = len(r.prompt)
            self._emit(r, row, [int(rng.integers(0, self.cfg.model.vocab))])
            r.drafts = []
            rids.append(rid)
        self._propose(batch_native=True)
        return rids

    def _fill_caches_random(self, seed: int) -> None:
        gen = torch.Generator(device=self.device).manual_seed(seed) if torch.device(self.device).type == "cuda" \
            else torch.Generator().manual_seed(seed)

        def fill(x):
            if isinstance(x, torch.Tensor):
                if x.dtype in (torch.bfloat16, torch.float16, torch.float32):
                    x.normal_(0.0, 1.0, generator=gen)
                elif x.dtype == torch.uint8:  # packed rows (e2m1 / e4m3 / bf16 bytes): small finite values
                    x.random_(0, 0x40, generator=gen)
                elif x.dtype == torch.float8_e4m3fn:
                    x.view(torch.uint8).random_(0, 0x40, generator=gen)
            elif isinstance(x, dict):
                for v in x.values():
                    fill(v)
            elif isinstance(x, (list, tuple)):
                for v in x:
                    fill(v)
            elif hasattr(x, "__dict__"):
                for name, v in vars(x).items():
                    if "state" in name:  # recurrent (GDN) states start from zero, as after a real prefill reset
                        if isinstance(v, torch.Tensor):
                            v.zero_()
                        continue
                    fill(v)

        fill(self.caches)
        if self.dcaches is not None:
            fill(self.dcaches)

    def abort_request(self, rid: str) -> bool:
        """Stop a request; a running one leaves at this step boundary. False if unknown or done."""
        r = self.prefilling
        if r is not None and r.rid == rid:
            self._drain()
            self.prefilling = None
            self.pool.release(r.blocks)
            r.blocks = []
            if r.slot:
                self._free_slots.append(r.slot)
                r.slot = 0
            r.finished, r.finish_reason = True, "abort"
            self.finished[rid] = r
            return True
        for i, r in enumerate(self.waiting):
            if r.rid == rid:
                self.waiting.pop(i)
                r.finished, r.finish_reason = True, "abort"
                self.finished[rid] = r
                return True
        for r in self.running:
            if r.rid == rid and not r.finished:
                self._drain()
                r.finished, r.finish_reason = True, "abort"
                self._retire()
                return True
        return False

    def poll(self, rid: str):
        """(new output tokens since the last poll, finished, finish_reason) of a request."""
        r = self.finished.get(rid)
        if r is None:
            r = next((q for q in self.running if q.rid == rid), None)
        if r is None:
            r = next((q for q in self.waiting if q.rid == rid), None)
        if r is None and self.prefilling is not None and self.prefilling.rid == rid:
            r = self.prefilling
        if r is None:
            raise KeyError(rid)
        new = r.output[r.polled:]
        r.polled = len(r.output)
        return new, r.finished, r.finish_reason

    def _corpus_caches(self) -> list:
        return [c for c in (getattr(self.proposer, "suffix_cache", None),
                            getattr(self.async_proposer, "suffix_cache", None)) if c is not None]

    def save_corpus(self, path: Optional[str] = None) -> int:
        """Snapshot the proposer's suffix corpus (every held sequence, oldest first) to `path` (default:
        SUFFIX_HYBRID_CORPUS_FILE), written to a temporary file and renamed over it; returns the count."""
        path = path or self.corpus_file
        caches = self._corpus_caches()
        if not path or not caches:
            raise RuntimeError("save_corpus needs a path and a suffix-corpus proposer")
        return int(caches[0].save(path))

    def load_corpus(self, path: Optional[str] = None) -> int:
        """Add a snapshot's sequences to every suffix corpus of the proposers (the file is checked whole
        before anything is added; the corpus bounds apply); returns the count."""
        path = path or self.corpus_file
        caches = self._corpus_caches()
        if not path or not caches:
            raise RuntimeError("load_corpus needs a path and a suffix-corpus proposer")
        n = 0
        for c in caches:
            n = int(c.load(path))
        return n

    def warm_start(self, sequences) -> int:
        """Pre-fill the proposer's suffix corpus with token histories (same path as a departing request)."""
        caches = self._corpus_caches()
        if not caches:
            raise RuntimeError(f"warm start needs a suffix-corpus proposer (method {self.cfg.spec.method!r})")
        n = 0
        for seq in sequences:
            toks = [int(t) for t in seq]
            for c in caches:
                c.add_sequence(toks)
            n += 1
        return n

    @torch.no_grad()
    def features(self, seq) -> torch.Tensor:
        """The target's pre-norm hidden state at every position of a token sequence (scratch KV blocks and
        the scratch recurrent slot; running requests are unaffected)."""
        self._drain()
        seq = np.asarray(seq, dtype=np.int64)
        blocks = self.pool.allocate(blocks_for(len(seq), self.block_size))
        try:
            return self.runner.prefill([seq], [blocks], [0], features=True)
        finally:
            self.pool.release(blocks)

    def idle_step(self) -> bool:
        """One bounded slice of idle-time work (online draft-head tuning); False when nothing ran."""
        if self.tuner is None or self.has_work():
            return False
        return self.tuner.micro_step()

    def readout(self, prompt, rows: torch.Tensor) -> List[float]:
        """Score one prompt: rows [R, H] . final hidden state at the prompt's last position (fp32).

        Runs between decode steps on scratch KV blocks (released afterwards) and the scratch recurrent
        slot, so running requests are unaffected.  Used by the decision endpoint."""
        self._drain()
        prompt = np.asarray(prompt, dtype=np.int64)
        if len(prompt) == 0 or len(prompt) > self.max_model_len:
            raise ValueError("decision input must fit the model length without truncation")
        blocks = self.pool.allocate(blocks_for(len(prompt), self.block_size))
        try:
            hid = self.runner.prefill([prompt], [blocks], [0], hidden_only=True)
            return (hid.float() @ rows.to(hid.device).float().t())[0].tolist()
        finally:
            self.pool.release(blocks)

    def proposer_stats(self) -> dict:
        get = getattr(self.proposer, "get_stats", None)
        return dict(get()) if get else {}

    def has_work(self) -> bool:
        local = bool(self.waiting or self.running or self.prefilling is not None or self._pipe is not None)
        if self.dp > 1:  # data-parallel attention: every rank steps while any rank has work
            return bool(self._dp_gather([int(local)]).max())
        return local

    def _dp_gather(self, values) -> torch.Tensor:
        """[world, len(values)] of every rank's values (control plane, gloo)."""
        import torch.distributed as dist

        st = pstate.get()
        t = torch.tensor(values, dtype=torch.long)
        out = [torch.empty_like(t) for _ in range(st.world)]
        dist.all_gather(out, t, group=st.cpu_group)
        return torch.stack(out)

    def _dp_step(self) -> StepStats:
        """Lockstep step under data-parallel attention: all ranks run the same kind of step with the same
        padded shapes (every MoE layer exchanges equal token counts), idle ranks run padding only."""
        free = self.cfg.max_num_seqs - len(self.running)
        batch = self._select_prefill(free) if (self.waiting and free > 0) else []
        info = self._dp_gather([len(batch), sum(len(r.prompt) for r in batch), len(self.running)])
        if int(info[:, 0].max()) > 0:
            n_max = int(info[:, 0].max())
            t_max = int((info[:, 1] + (n_max - info[:, 0])).max())
            return self._prefill_step(0, batch=batch, pad=(n_max, t_max))
        if int(info[:, 2].max()) > 0:
            return self._decode_step(nb_min=int(info[:, 2].max()))
        return StepStats("idle", 0, 0, 0, 0.0, 0.0, 0.0)

    def step(self) -> StepStats:
        if self.dp > 1:
            return self._dp_step()
        # a long prompt's chunks alternate with decode steps of the running requests
        if self.prefilling is not None and (not self.running or self._last_kind != "chunk"):
            return self._chunk_step()
        free_rows = self.cfg.max_num_seqs - len(self.running) - (self.prefilling is not None)
        # a waiting request is prefilled once a row is free and the KV blocks not promised to running requests
        # cover it (otherwise the running ones decode on, without breaking the decode pipeline, until they do)
        if self.waiting and free_rows > 0 and (not self.running or
                                               self._reservation(self.waiting[0]) <= self._unclaimed_blocks()):
            if self._chunkable(self.waiting[0]):
                r0 = self.waiting[0]
                if not self.running and self._reservation(r0) > self._unclaimed_blocks():
                    raise MemoryError(f"request {r0.rid} needs {self._reservation(r0)} KV blocks, the pool has "
                                      f"{self.pool.free} free")
                if self.prefilling is None:
                    self._drain()
                    self.prefilling = self.waiting.pop(0)
                    return self._chunk_step()
            else:
                self._drain()
                batch = self._select_prefill(free_rows)
                if batch:
                    return self._prefill_step(0, batch)
        self._last_kind = "decode"
        decode = self._decode_step_async if self._async else self._decode_step
        sp = self.step_profiler
        if sp is not None:
            sp.before("decode", len(self.running))
            try:
                return decode()
            finally:
                sp.after()
        return decode()

    def generate(self, prompts, max_new_tokens: int = 128) -> List[List[int]]:
        rids = [self.add_request(p, max_new_tokens) for p in prompts]
        while self.has_work():
            self.step()
        return [self.finished[r].output for r in rids]

    def spec_stats(self) -> dict:
        dec = [s for s in self.stats if s.kind == "decode"]
        steps = sum(s.num_reqs for s in dec)
        emitted = sum(s.emitted for s in dec)
        return {
            "decode_steps": len(dec),
            "mean_accept_len": emitted / steps if steps else 0.0,
            "proposer_us_per_step": (sum(s.proposer_us for s in dec) / len(dec)) if dec else 0.0,
        }

    # ------------------------------------------------------------------ internals
    def _ensure_blocks(self, r: Request, upto_tokens: int) -> None:
        need = blocks_for(upto_tokens, self.block_size) - len(r.blocks)
        if need > 0:
            r.blocks.extend(self.pool.allocate(need))
        if r.blocks_np.shape[0] != len(r.blocks):  # the block-table row the decode steps copy
            r.blocks_np = np.asarray(r.blocks, dtype=np.int32)

    def _reservation(self, r: Request) -> int:
        """Blocks request r can ever hold: its prompt and every output token, plus the verify window's
        look-ahead (the decode step keeps blocks for committed + 2k + 2 positions)."""
        return blocks_for(len(r.prompt) + r.max_new_tokens + 2 * self.k + 2, self.block_size)

    def _unclaimed_blocks(self) -> int:
        """Free blocks not yet promised to a running request's remaining growth."""
        owed = sum(max(0, self._reservation(r) - len(r.blocks)) for r in self.running)
        if self.prefilling is not None:
            owed += max(0, self._reservation(self.prefilling) - len(self.prefilling.blocks))
        return self.pool.free - owed

    def _chunkable(self, r: Request) -> bool:
        """Whether r's prompt is prefilled in chunks (longer than the prefill budget, attention-only model,
        no data-parallel lockstep)."""
        return (self.cfg.chunked_prefill and len(r.prompt) > self.cfg.max_prefill_tokens and self.dp == 1
                and not self.runner.recurrent)

    def _chunk_step(self) -> StepStats:
        """Prefill the next max_prefill_tokens of the long prompt; its last chunk makes it a running request."""
        t0 = time.perf_counter()
        r = self.prefilling
        self._drain()
        if not r.slot:
            r.slot = self._free_slots.pop()
        s = r.prefilled
        e = min(len(r.prompt), s + self.cfg.max_prefill_tokens)
        final = e == len(r.prompt)
        self._ensure_blocks(r, e + (2 * self.k + 2 if final else 0))
        first, natives = self.runner.prefill([r.prompt[s:e]], [r.blocks], [r.slot], starts=[s],
                                             follow=[None if final else int(r.prompt[e])], drafts=final)
        r.prefilled = e
        self._last_kind = "chunk"
        prop_us = 0.0
        if final:
            self.prefilling = None
            row = len(self.running)
            self.running.append(r)
            self.tokens[row, :len(r.prompt)] = r.prompt
            r.committed = len(r.prompt)
            self._emit(r, row, [int(first[0])])
            r.drafts = [int(x) for x in natives[0][: self.k]]
        t1 = time.perf_counter()
        if final:
            prop_us = self._propose(batch_native=True)
            self._retire()
        st = StepStats("prefill", 1, 1 if final else 0, 0, (t1 - t0) * 1e3, 0.0, prop_us)
        self.stats.append(st)
        return st

    def _select_prefill(self, free_rows: int) -> list:
        """Waiting requests to prefill, in arrival order, within the prefill token budget and the KV blocks
        that are not promised to running requests (each admitted request reserves its own maximum, so the
        pool never runs dry mid-generation; a request that does not fit waits for others to finish)."""
        batch, budget = [], self.cfg.max_prefill_tokens
        blocks = self._unclaimed_blocks()
        while self.waiting and len(batch) < free_rows:
            r = self.waiting[0]
            if batch and len(r.prompt) > budget:
                break
            need = self._reservation(r)
            if need > blocks:
                if not batch and not self.running:
                    raise MemoryError(f"request {r.rid} needs {need} KV blocks, the pool has {self.pool.free} free")
                break
            self.waiting.pop(0)
            batch.append(r)
            budget -= len(r.prompt)
            blocks -= need
        return batch

    def _prefill_step(self, free_rows: int, batch: Optional[list] = None, pad: Optional[tuple] = None) -> StepStats:
        """Prefill a batch; pad = (prompts, tokens) adds padding prompts on the scratch block and slot so every
        data-parallel rank runs the same shapes (their results are dropped)."""
        t0 = time.perf_counter()
        if batch is None:
            batch = self._select_prefill(free_rows)
        for r in batch:
            self._ensure_blocks(r, len(r.prompt) + 2 * self.k + 2)
            r.slot = self._free_slots.pop()
        prompts = [r.prompt for r in batch]
        tables = [r.blocks for r in batch]
        slots = [r.slot for r in batch]
        if pad is not None:
            n_pad = pad[0] - len(batch)
            left = pad[1] - sum(len(p) for p in prompts)
            for j in range(n_pad):
                ln = left - (n_pad - 1 - j) if j == 0 else 1
                left -= ln
                prompts.append(np.zeros(ln, dtype=np.int64))
                tables.append([0] * blocks_for(ln + 2 * self.k + 2, self.block_size))
                slots.append(0)
        first, natives = self.runner.prefill(prompts, tables, slots)
        for i, r in enumerate(batch):
            row = len(self.running)
            self.running.append(r)
            self.tokens[row, :len(r.prompt)] = r.prompt
            r.committed = len(r.prompt)
            self._emit(r, row, [int(first[i])])
            r.drafts = [int(x) for x in natives[i][: self.k]]
        t1 = time.perf_counter()
        prop_us = self._propose(batch_native=True)
        self._retire()
        st = StepStats("prefill", len(batch), len(batch), 0, (t1 - t0) * 1e3, 0.0, prop_us)
        self.stats.append(st)
        return st

    def _emit(self, r: Request, row: int, toks: List[int]) -> None:
        room = r.max_new_tokens - len(r.output)
        toks = toks[:room]
        stopped = False
        if r.stop_ids:
            for j, t in enumerate(toks):
                if t in r.stop_ids:
                    toks, stopped = toks[: j + 1], True
                    break
        n0 = r.history_len
        self.tokens[row, n0:n0 + len(toks)] = toks
        r.output.extend(toks)
        r.next_token = toks[-1] if toks else r.next_token
        if stopped:
            r.finished, r.finish_reason = True, "stop"
        elif len(r.output) >= r.max_new_tokens or r.history_len + 2 * self.k + 2 + 2 * self._lag >= self.max_model_len:
            r.finished, r.finish_reason = True, "length"

    def _propose(self, batch_native: bool) -> float:
        """Replace each running request's drafts by the proposer's choice."""
        t0 = time.perf_counter_ns()
        n = len(self.running)
        if n == 0 or self.k == 0 or (self.proposer is None and self.cfg.spec.method != "external"):
            return 0.0
        method = self.cfg.spec.method
        ids = [r.rid for r in self.running]
        counts = np.fromiter((r.history_len for r in self.running), dtype=np.int64, count=n)
        if method == "hybrid":
            acc = [r.accepted_prev for r in self.running]
            drafts = self.proposer.mix_numpy(ids, counts, self.tokens, [r.drafts for r in self.running],
                                             acc if any(a >= 0 for a in acc) else None)
        elif method == "suffix":
            packed, widths = self.proposer.propose_suffix_only(ids, np.arange(n, dtype=np.int64), counts,
                                                               self.tokens)
            drafts = [packed[i, : widths[i]].tolist() for i in range(n)]
        elif method == "external":
            drafts = self.external_proposer(self.running) if self.external_proposer else [[] for _ in range(n)]
            # A caller's lists may be reused or mutated later and may hold NumPy ints: copy them.
            for r, d in zip(self.running, drafts):
                r.drafts = [int(x) for x in d]
            return (time.perf_counter_ns() - t0) / 1e3
        else:  # ngram
            drafts = self.proposer.propose([[1]] * n, counts, self.tokens)
        for r, d in zip(self.running, drafts):  # the native proposers return fresh lists of Python ints
            r.drafts = d if type(d) is list else [int(x) for x in d]
        return (time.perf_counter_ns() - t0) / 1e3

    def _decode_step(self, nb_min: int = 0) -> StepStats:
        t0 = time.perf_counter()
        n = len(self.running)
        if n == 0 and nb_min == 0:
            return StepStats("idle", 0, 0, 0, 0.0, 0.0, 0.0)
        k, W = self.k, self.k + 1
        win = np.full((n, W), 0, dtype=np.int64)
        seq = np.empty(n, dtype=np.int64)
        mb = self.max_blocks_per_seq
        bt = np.zeros((n, mb), dtype=np.int32)
        slots = np.fromiter((r.slot for r in self.running), dtype=np.int64, count=n)
        for i, r in enumerate(self.running):
            self._ensure_blocks(r, r.committed + 2 * k + 2)
            b = r.blocks_np
            bt[i, :b.shape[0]] = b
        width = W
        if n:
            win[:, 0] = np.fromiter((r.next_token for r in self.running), dtype=np.int64, count=n)
            seq[:] = np.fromiter((r.committed for r in self.running), dtype=np.int64, count=n)
            if k:
                win[:, 1:] = [r.drafts[:k] if len(r.drafts) >= k else r.drafts + [-1] * (k - len(r.drafts))
                              for r in self.running]
                if self.adaptive_width and nb_min == 0:
                    # Verify only as wide as the longest real draft (-1 pads never match a target token).
                    real = (win[:, 1:] >= 0).cumprod(axis=1).sum(axis=1)
                    width = 1 + int(real.max())
        t1 = time.perf_counter()
        out, acc, nat = self.runner.decode(n, win, seq, bt, slots, nb_min=nb_min, width=width)
        t2 = time.perf_counter()
        emitted = 0
        accepted = 0
        acc_l, out_l = acc[:n].tolist(), out[:n].tolist()  # one conversion per step, not per row
        nat_l = nat[:n, :k].tolist() if self.draft is not None and k > 0 else None
        for i, r in enumerate(self.running):
            a = acc_l[i]
            toks = out_l[i][: a + 1]
            r.committed += a + 1
            r.accepted_prev = a
            self._emit(r, i, toks)
            emitted += min(a + 1, len(toks))
            accepted += a
            if nat_l is not None:
                r.drafts = nat_l[i]
        prop_us = self._propose(batch_native=False)
        self._retire()
        t3 = time.perf_counter()
        st = StepStats("decode", n, emitted, accepted, (t2 - t1) * 1e3, (t3 - t2 + t1 - t0) * 1e3, prop_us)
        self.stats.append(st)
        self.telemetry.record(self, st)
        return st

    # ------------------------------------------------------------------ async scheduling
    def _take(self, out, acc, used, real, pub=None) -> tuple:
        """Commit one collected pipelined step: emit for rows still running; (emitted, accepted)."""
        emitted = accepted = 0
        for i, r in enumerate(self.running):
            a = int(acc[i])
            if r.finished:  # finished at an earlier step: the lagged step's tokens are dropped
                continue
            toks = out[i, : a + 1].tolist()
            r.committed += a + 1
            r.accepted_prev = a
            self._emit(r, i, toks)
            emitted += min(a + 1, len(toks))
            accepted += a
        if self._trace_verify[0] > 0:
            self._trace_verify[0] -= 1
            for i, r in enumerate(self.running):
                w = self.k
                graded = [int(x) for x in used[i, 1:1 + w]]
                p = pub[i] if pub is not None else graded
                m = sum(1 for x, y in zip(p, graded) if x == y)
                logger.warning("VTRACE2 rid=%r w=%d pubmatch=%d/%d graded=%s pub=%s accrow=%s nacc=%d real=%d", r.rid,
                               w, m, w, graded[:8], list(p)[:8], out[i, :8].tolist(), int(acc[i]), int(real[i]))
        return emitted, accepted

    def _drain(self) -> None:
        """Collect the in-flight pipelined step (before the running set changes)."""
        if self._pipe is None:
            return
        n = len(self.running)
        out, acc, nat, used, real = self.runner.collect(self._pipe["parity"], n)
        em, ac = self._take(out, acc, used, real)
        self._pipe = None
        if self.draft is not None:
            for i, r in enumerate(self.running):
                r.drafts = nat[i, : self.k].tolist()
        self._propose(batch_native=False)  # host drafts for the next synchronous step
        st = StepStats("decode", n, em, ac, 0.0, 0.0, 0.0)
        self.stats.append(st)
        self.telemetry.record(self, st)
        self._retire()

    def _decode_step_async(self) -> StepStats:
        """Pipelined decode: launch step N (window advanced on the device from step N-1's results and a
        candidate looked up on the host from the history before step N-1), then collect step N-1.

        Reference behaviour: suffix_hybrid/async_spec.py:1-120 (lag-1 host lookup, device resolve,
        hybrid replacement threshold); here the resolve checks the candidate against the in-flight
        step's accepted tokens, so no device copy of the token history is needed."""
        t0 = time.perf_counter()
        n = len(self.running)
        if n == 0:
            self._drain()
            return StepStats("idle", 0, 0, 0, 0.0, 0.0, 0.0)
        ids = [r.rid for r in self.running]
        if self._pipe is not None and self._pipe["rows"] != ids:
            self._drain()
            return self._decode_step()
        if self._pipe is None and not self.runner.has_graph(n):
            return self._decode_step()  # captures the bucket's graph synchronously
        k, W = self.k, self.k + 1
        mb = self.max_blocks_per_seq
        bt = np.zeros((n, mb), dtype=np.int32)
        slots = np.fromiter((r.slot for r in self.running), dtype=np.int64, count=n)
        for i, r in enumerate(self.running):
            self._ensure_blocks(r, r.committed + 2 * k + 2 + 2 * self._lag)
            b = r.blocks_np
            bt[i, :b.shape[0]] = b
        if self._pipe is None:  # pipeline start: host window (drafts from the synchronous proposer)
            win = np.full((n, W), -1, dtype=np.int64)
            seq = np.fromiter((r.committed for r in self.running), dtype=np.int64, count=n)
            for i, r in enumerate(self.running):
                win[i, 0] = r.next_token
                d = r.drafts[:k]
                win[i, 1:1 + len(d)] = d
            self.runner.launch(0, n, bt, slots, win=win, seq=seq, cand_len=self._cand_len)
            self._pipe = {"parity": 0, "rows": ids}
            st = StepStats("launch", n, 0, 0, 0.0, (time.perf_counter() - t0) * 1e3, 0.0)
            self.stats.append(st)
            return st
        tp = time.perf_counter_ns()
        counts = np.fromiter((r.history_len for r in self.running), dtype=np.int64, count=n)
        cand, clen = self.async_proposer.propose_suffix_only(ids, np.arange(n, dtype=np.int64), counts, self.tokens)
        prop_us = (time.perf_counter_ns() - tp) / 1e3
        p = self._pipe["parity"]
        q = p ^ 1
        self.runner.launch(q, n, bt, slots, cand=cand, clen=np.asarray(clen, dtype=np.int32), hyb_min=self._hyb_min,
                           cand_len=self._cand_len)
        if self._trace_sched[0] > 0:
            self._trace_sched[0] -= 1
            logger.warning("SCHEDTRACE step rows=%d host_widths=%s", n,
                           [int(min(k, max(int(c) - 1, 0))) for c in clen][:16])
        t1 = time.perf_counter()
        out, acc, nat, used, real = self.runner.collect(p, n)
        t2 = time.perf_counter()
        em, ac = self._take(out, acc, used, real, pub=self._pipe.get("pub"))
        self._pipe = {"parity": q, "rows": ids, "pub": [list(cand[i, 1:1 + k]) for i in range(n)]}
        if any(r.finished for r in self.running):
            self._drain()
        st = StepStats("decode", n, em, ac, (t2 - t1) * 1e3, (t1 - t0) * 1e3, prop_us)
        self.stats.append(st)
        self.telemetry.record(self, st)
        return st

    def _retire(self) -> None:
        """Move finished requests out; back-fill their token rows."""
        i = 0
        while i < len(self.running):
            r = self.running[i]
            if not r.finished:
                i += 1
                continue
            if self.tuner is not None and r.finish_reason != "abort":
                self.tuner.capture(r.rid, np.concatenate([np.asarray(r.prompt, dtype=np.int64),
                                                          np.asarray(r.output, dtype=np.int64)]))
            self.pool.release(r.blocks)
            r.blocks = []
            if r.slot:
                self._free_slots.append(r.slot)
                r.slot = 0
            self.finished[r.rid] = r
            last = len(self.running) - 1
            if i != last:
                mv = self.running[last]
                self.tokens[i, : mv.history_len] = self.tokens[last, : mv.history_len]
                self.running[i] = mv
            self.running.pop()
