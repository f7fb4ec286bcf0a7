"""Async front end: LLMEngine stepped in a dedicated thread, fed by a control queue.

Every mutation of engine state (add, abort, warm start, shutdown) is an
``EngineOp`` applied between steps in the engine thread, in arrival order.
With tensor parallelism (one process per GPU) rank 0 owns the queue: each
iteration it broadcasts the batch of pending ops over the gloo control
group and every rank applies the same ops before the same ``step()``, so the
ranks' engines stay in lockstep (the reference's TP ranks agree by broadcast
too, reference: suffix_hybrid/wrap_v2.py:1680-1707).  Ranks other than 0 run
``worker_loop()``.

Consumers get tokens through per-request asyncio queues fed after each step
(streaming) or await the whole result.
"""
from __future__ import annotations

import asyncio
import logging
import queue
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

logger = logging.getLogger("suffix_hybrid.serve")


@dataclass
class EngineOp:
    kind: str  # "add" | "abort" | "warm" | "corpus_save" | "readout" | "stop"
    rid: str = ""
    prompt: List[int] = field(default_factory=list)
    max_new_tokens: int = 0
    stop_token_ids: List[int] = field(default_factory=list)
    sequences: List[List[int]] = field(default_factory=list)
    payload: Any = None  # readout rows (single-rank engines only)


class AsyncEngine:
    def __init__(self, engine, rank: int = 0, world: int = 1, cpu_group=None):
        self.engine = engine
        self.rank, self.world, self.cpu_group = rank, world, cpu_group
        self._ops: "queue.Queue[EngineOp]" = queue.Queue()
        self._streams: Dict[str, tuple] = {}  # rid -> (loop, asyncio.Queue)
        self._futures: Dict[str, tuple] = {}  # op id -> (loop, future) for warm start results
        self._lock = threading.Lock()
        self._thread: Optional[threading.Thread] = None
        self._running = False
        self._counter = 0
        from ..parallel.health import RankHealth

        # lockstep ranks share a failure flag in the rendezvous store, tested every 8th step (one store round
        # trip); a failed collective in between is explained from the same flag
        self.health = RankHealth.from_process_group(every=8) if world > 1 else RankHealth()
        self.metrics = {"requests_total": 0, "requests_finished": 0, "requests_aborted": 0,
                        "generated_tokens_total": 0, "decode_steps_total": 0, "prefill_steps_total": 0,
                        "step_seconds_total": 0.0, "warm_start_sequences_total": 0}

    # ------------------------------------------------------------------ control (any thread)
    def start(self) -> None:
        self._running = True
        self._thread = threading.Thread(target=self._loop, name="engine", daemon=True)
        self._thread.start()

    def shutdown(self) -> None:
        self._ops.put(EngineOp("stop"))
        if self._thread is not None:
            self._thread.join(timeout=60)
        e = self.engine
        if getattr(e, "corpus_file", None) and e._corpus_caches():  # keep the corpus for the next start
            try:
                logger.warning("suffix corpus saved to %s: %d sequences", e.corpus_file, e.save_corpus())
            except RuntimeError as err:
                logger.warning("suffix corpus not saved: %s", err)

    def new_rid(self) -> str:
        with self._lock:
            self._counter += 1
            return f"cmpl-{self._counter}-{int(time.time() * 1e3)}"

    async def generate(self, prompt: List[int], max_new_tokens: int, stop_token_ids=None, rid: Optional[str] = None):
        """Async generator of (new_tokens, finished, finish_reason) updates for one request."""
        rid = rid or self.new_rid()
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        with self._lock:
            self._streams[rid] = (loop, q)
        self._ops.put(EngineOp("add", rid, [int(t) for t in prompt], int(max_new_tokens),
                               [int(t) for t in (stop_token_ids or [])]))
        try:
            while True:
                item = await q.get()
                if isinstance(item, Exception):
                    raise item
                yield item
                if item[1]:
                    return
        finally:
            with self._lock:
                live = self._streams.pop(rid, None)
            if live is not None:
                self._ops.put(EngineOp("abort", rid))  # consumer went away early

    def abort(self, rid: str) -> None:
        self._ops.put(EngineOp("abort", rid))

    async def warm_start(self, sequences) -> int:
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        key = f"warm-{self.new_rid()}"
        with self._lock:
            self._futures[key] = (loop, fut)
        self._ops.put(EngineOp("warm", key, sequences=[[int(t) for t in s] for s in sequences]))
        return await fut

    async def save_corpus(self, path: Optional[str] = None) -> int:
        """Snapshot the suffix corpus on the engine thread (rank 0 writes the file); returns the count."""
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        key = f"corpus-{self.new_rid()}"
        with self._lock:
            self._futures[key] = (loop, fut)
        self._ops.put(EngineOp("corpus_save", key, payload=path))
        return await fut

    async def readout(self, prompt: List[int], rows) -> List[float]:
        """Score one prompt on the engine thread (LLMEngine.readout); single-rank engines only."""
        if self.world > 1:
            raise ValueError("the decision endpoint runs on single-rank engines")
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        key = f"readout-{self.new_rid()}"
        with self._lock:
            self._futures[key] = (loop, fut)
        self._ops.put(EngineOp("readout", key, sequences=[[int(t) for t in prompt]], payload=rows))
        return await fut

    async def sft_call(self, kind: str, payload) -> Any:
        """Run an SFT control op on the engine thread (every rank, in step order): "sft_begin" (returns the
        run id; training then proceeds between serving steps) or "sft_load"."""
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        key = f"{kind}-{self.new_rid()}"
        with self._lock:
            self._futures[key] = (loop, fut)
        self._ops.put(EngineOp(kind, key, payload=payload))
        return await fut

    def stats(self) -> dict:
        e = self.engine
        out = dict(self.metrics)
        out.update({"running": len(e.running), "waiting": len(e.waiting),
                    "prefilling": int(getattr(e, "prefilling", None) is not None)})
        tier = getattr(e, "host_tier", None)
        if tier is not None:
            out["host_kv_hit_rate"] = tier.hit_rate()
        out.update(e.spec_stats())
        out["proposer"] = e.proposer_stats()
        return out

    # ------------------------------------------------------------------ engine thread
    def _drain(self, block: bool) -> List[EngineOp]:
        ops = []
        try:
            ops.append(self._ops.get(timeout=0.05) if block else self._ops.get_nowait())
            while True:
                ops.append(self._ops.get_nowait())
        except queue.Empty:
            pass
        return ops

    def _sync_ops(self, ops: List[EngineOp]) -> List[EngineOp]:
        if self.world <= 1:
            return ops
        import torch.distributed as dist

        self.health.check()  # a peer that recorded a failure is not waited for
        box = [ops]
        try:
            dist.broadcast_object_list(box, src=0, group=self.cpu_group)
        except Exception as err:  # a peer left: the collective's timeout or a closed connection
            raise self.health.explain(err) from err
        return box[0]

    def _apply(self, ops: List[EngineOp]) -> bool:
        e = self.engine
        for op in ops:
            if op.kind == "stop":
                return False
            if op.kind == "add":
                try:
                    e.add_request(op.prompt, op.max_new_tokens, rid=op.rid, stop_token_ids=op.stop_token_ids)
                    self.metrics["requests_total"] += 1
                except Exception as ex:  # invalid request: report to its stream
                    self._push(op.rid, ex)
            elif op.kind == "abort":
                if e.abort_request(op.rid):
                    self.metrics["requests_aborted"] += 1
            elif op.kind in ("sft_begin", "sft_load", "sft_step"):
                try:
                    if e.sft is None:
                        raise RuntimeError("SFT is not enabled (SUFFIX_SFT=1)")
                    if op.kind == "sft_begin":
                        res = e.sft.begin(**op.payload)
                    elif op.kind == "sft_load":
                        res = e.sft.load(op.payload)
                    else:
                        res = e.sft.micro()
                    self._resolve(op.rid, res)
                except Exception as ex:
                    self._resolve(op.rid, ex)
            elif op.kind == "tune":
                e.idle_step()
            elif op.kind == "readout":
                try:
                    self._resolve(op.rid, e.readout(op.sequences[0], op.payload))
                except Exception as ex:
                    self._resolve(op.rid, ex)
            elif op.kind == "warm":
                try:
                    n = e.warm_start(op.sequences)
                    self.metrics["warm_start_sequences_total"] += n
                    self._resolve(op.rid, n)
                except Exception as ex:
                    self._resolve(op.rid, ex)
            elif op.kind == "corpus_save" and self.rank == 0:  # the ranks' corpora are identical in lockstep
                try:
                    self._resolve(op.rid, e.save_corpus(op.payload))
                except Exception as ex:
                    self._resolve(op.rid, ex)
        return True

    def _push(self, rid: str, item: Any) -> None:
        if self.rank != 0:
            return
        with self._lock:
            ent = self._streams.get(rid)
        if ent is not None:
            loop, q = ent
            loop.call_soon_threadsafe(q.put_nowait, item)

    def _resolve(self, key: str, value: Any) -> None:
        if self.rank != 0:
            return
        with self._lock:
            ent = self._futures.pop(key, None)
        if ent is None:
            return
        loop, fut = ent

        def done():
            if not fut.done():
                (fut.set_exception if isinstance(value, Exception) else fut.set_result)(value)

        loop.call_soon_threadsafe(done)

    def _publish(self) -> None:
        """Hand each stream its new tokens; drop finished requests from the engine's table."""
        e = self.engine
        with self._lock:
            items = list(self._streams.items())
        for rid, (loop, q) in items:
            try:
                new, fin, why = e.poll(rid)
            except KeyError:
                continue
            if not (new or fin):
                continue
            self.metrics["generated_tokens_total"] += len(new)
            if fin:
                self.metrics["requests_finished"] += 1
                with self._lock:
                    self._streams.pop(rid, None)
                e.finished.pop(rid, None)
            loop.call_soon_threadsafe(q.put_nowait, (new, fin, why))
        for rid in list(e.finished):  # no consumer (other TP ranks, aborted streams)
            e.finished.pop(rid, None)

    def _loop(self) -> None:
        e = self.engine
        alive = True
        while alive:
            idle = not e.has_work()
            ops = self._drain(block=idle) if self.rank == 0 else []
            sft = getattr(e, "sft", None)
            if sft is not None and self.rank == 0 and sft.wants_step(busy=not idle):
                ops.append(EngineOp("sft_step"))  # one optimizer step of the active run, on every rank
            tuner = getattr(e, "tuner", None)
            if tuner is not None and self.rank == 0:
                if not idle or ops:
                    tuner.note_work()
                elif tuner.wants_step():
                    ops.append(EngineOp("tune"))  # every rank runs the same idle micro-step
            if self.world > 1:
                ops = self._sync_ops(ops)
            alive = self._apply(ops)
            if not alive:
                break
            if not e.has_work():
                if self.world > 1 and not ops:
                    time.sleep(0.001)
                continue
            t0 = time.perf_counter()
            try:
                st = e.step()
            except Exception as ex:  # a failed step fails every live request
                logger.exception("engine step failed")
                self.health.report(f"engine step failed: {ex!r}")  # the peers stop instead of waiting
                with self._lock:
                    rids = list(self._streams)
                for rid in rids:
                    self._push(rid, RuntimeError(f"engine step failed: {ex!r}"))
                raise
            self.metrics["step_seconds_total"] += time.perf_counter() - t0
            if st.kind == "decode":
                self.metrics["decode_steps_total"] += 1
            elif st.kind == "prefill":
                self.metrics["prefill_steps_total"] += 1
            self._publish()
        self._running = False

    def worker_loop(self) -> None:
        """Ranks != 0 under TP: apply rank 0's ops and step in lockstep until "stop"."""
        self._loop()
