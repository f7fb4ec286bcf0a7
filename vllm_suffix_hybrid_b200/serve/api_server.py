"""OpenAI-style HTTP API over AsyncEngine (FastAPI).

Routes:
  GET  /health, /v1/models
  POST /v1/completions        prompt: str | list[int]; max_tokens; stream; stop_token_ids
  POST /v1/chat/completions   messages (chat template of the tokenizer, else a plain role template)
  GET  /metrics               Prometheus text format (counters and gauges of the engine)
  GET  /v1/spec_stats         speculative-decoding and proposer statistics (JSON)
  POST /debug/warm-start      {"sequences": [[ids...], ...]} -> {"ingested": N}; only with
                              SUFFIX_HYBRID_WARMSTART=1 (the reference's route and gate,
                              reference: suffix_hybrid/warmstart.py)
  POST /debug/corpus-save     {"path": optional} -> {"saved": N, "path": p}: snapshot of the suffix
                              corpus (default path SUFFIX_HYBRID_CORPUS_FILE); same gate
Decoding is greedy (the verify step is the greedy accept run); a request
with temperature > 0 is rejected with 400.
"""
from __future__ import annotations

import json
import os
import time
from typing import Any, Dict, List

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse


def _err(code: int, msg: str) -> JSONResponse:
    return JSONResponse(status_code=code, content={"error": {"message": msg, "type": "invalid_request_error"}})


def build_app(aeng, tokenizer, model_name: str) -> FastAPI:
    app = FastAPI(title="vllm-suffix-hybrid-b200")
    created = int(time.time())
    eos = getattr(tokenizer, "eos_token_id", None)

    def prompt_ids(p) -> List[int]:
        if isinstance(p, str):
            return tokenizer.encode(p)
        if isinstance(p, list) and all(isinstance(t, int) for t in p):
            return list(p)
        raise ValueError("prompt must be a string or a list of token ids")

    def params(body: Dict[str, Any]):
        if float(body.get("temperature", 0.0) or 0.0) > 0.0:
            raise ValueError("only greedy decoding (temperature 0) is supported")
        max_tokens = int(body.get("max_tokens", body.get("max_completion_tokens", 16)) or 16)
        stop_ids = list(body.get("stop_token_ids") or [])
        if eos is not None and not body.get("ignore_eos", False):
            stop_ids.append(int(eos))
        return max_tokens, stop_ids

    async def run(ids, max_tokens, stop_ids, stream: bool, make_chunk, make_final):
        rid = aeng.new_rid()
        gen = aeng.generate(ids, max_tokens, stop_ids, rid=rid)
        if stream:
            async def sse():
                out, why = [], ""
                async for new, fin, why in gen:
                    out.extend(new)
                    if new:
                        yield "data: " + json.dumps(make_chunk(rid, new, None)) + "\n\n"
                yield "data: " + json.dumps(make_chunk(rid, [], why or "length")) + "\n\n"
                yield "data: [DONE]\n\n"

            return StreamingResponse(sse(), media_type="text/event-stream")
        out, why = [], ""
        async for new, fin, why in gen:
            out.extend(new)
        return JSONResponse(make_final(rid, ids, out, why or "length"))

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "created": created,
                                            "owned_by": "vllm-suffix-hybrid-b200"}]}

    @app.post("/v1/completions")
    async def completions(request: Request):
        try:
            body = await request.json()
            ids = prompt_ids(body.get("prompt", ""))
            max_tokens, stop_ids = params(body)
        except Exception as ex:
            return _err(400, str(ex))

        def chunk(rid, new, why):
            return {"id": rid, "object": "text_completion", "created": int(time.time()), "model": model_name,
                    "choices": [{"index": 0, "text": tokenizer.decode(new), "token_ids": new,
                                 "finish_reason": why}]}

        def final(rid, ids_, out, why):
            return {"id": rid, "object": "text_completion", "created": int(time.time()), "model": model_name,
                    "choices": [{"index": 0, "text": tokenizer.decode(out), "token_ids": out, "finish_reason": why}],
                    "usage": {"prompt_tokens": len(ids_), "completion_tokens": len(out),
                              "total_tokens": len(ids_) + len(out)}}

        try:
            return await run(ids, max_tokens, stop_ids, bool(body.get("stream", False)), chunk, final)
        except ValueError as ex:
            return _err(400, str(ex))

    @app.post("/v1/chat/completions")
    async def chat(request: Request):
        try:
            body = await request.json()
            msgs = body.get("messages")
            if not isinstance(msgs, list) or not msgs:
                raise ValueError("messages must be a non-empty list")
            ids = list(tokenizer.apply_chat_template(msgs))
            max_tokens, stop_ids = params(body)
        except Exception as ex:
            return _err(400, str(ex))

        def chunk(rid, new, why):
            return {"id": rid, "object": "chat.completion.chunk", "created": int(time.time()), "model": model_name,
                    "choices": [{"index": 0, "delta": {"role": "assistant", "content": tokenizer.decode(new)},
                                 "finish_reason": why}]}

        def final(rid, ids_, out, why):
            return {"id": rid, "object": "chat.completion", "created": int(time.time()), "model": model_name,
                    "choices": [{"index": 0, "message": {"role": "assistant", "content": tokenizer.decode(out)},
                                 "finish_reason": why}],
                    "usage": {"prompt_tokens": len(ids_), "completion_tokens": len(out),
                              "total_tokens": len(ids_) + len(out)}}

        try:
            return await run(ids, max_tokens, stop_ids, bool(body.get("stream", False)), chunk, final)
        except ValueError as ex:
            return _err(400, str(ex))

    @app.get("/v1/spec_stats")
    async def spec_stats():
        return aeng.stats()

    @app.get("/metrics")
    async def metrics():
        s = aeng.stats()
        lines = []
        for key in ("requests_total", "requests_finished", "requests_aborted", "generated_tokens_total",
                    "decode_steps_total", "prefill_steps_total", "warm_start_sequences_total"):
            lines += [f"# TYPE suffix_hybrid_{key} counter", f"suffix_hybrid_{key} {int(s[key])}"]
        lines += ["# TYPE suffix_hybrid_step_seconds_total counter",
                  f"suffix_hybrid_step_seconds_total {s['step_seconds_total']:.6f}"]
        for key in ("running", "waiting", "mean_accept_len", "proposer_us_per_step"):
            lines += [f"# TYPE suffix_hybrid_{key} gauge", f"suffix_hybrid_{key} {float(s.get(key, 0.0)):.6f}"]
        return PlainTextResponse("\n".join(lines) + "\n", media_type="text/plain; version=0.0.4")

    if os.environ.get("SUFFIX_HYBRID_WARMSTART", "0") == "1":
        @app.post("/debug/warm-start")
        async def warm_start(request: Request):
            try:
                body = await request.json()
            except Exception:
                return JSONResponse(status_code=400, content={"error": "bad json"})
            seqs = (body or {}).get("sequences")
            if not isinstance(seqs, list) or any(not isinstance(x, list) for x in seqs):
                return JSONResponse(status_code=400, content={"error": "sequences must be a list of token-id lists"})
            try:
                n = await aeng.warm_start(seqs)
            except Exception as ex:
                return JSONResponse(status_code=409, content={"error": str(ex)})
            return {"ingested": n}

        @app.post("/debug/corpus-save")
        async def corpus_save(request: Request):
            try:
                body = await request.json()
            except Exception:
                body = {}
            path = (body or {}).get("path") or getattr(aeng.engine, "corpus_file", None)
            if not isinstance(path, str) or not path:
                return JSONResponse(status_code=400, content={"error": "no path (body or SUFFIX_HYBRID_CORPUS_FILE)"})
            try:
                n = await aeng.save_corpus(path)
            except Exception as ex:
                return JSONResponse(status_code=409, content={"error": str(ex)})
            return {"saved": n, "path": path}

    if getattr(aeng.engine, "sft", None) is not None:
        from .sft_api import attach as attach_sft

        attach_sft(app, aeng, tokenizer)

    if os.environ.get("SUFFIX_PPLX_DECIDER", "0") == "1":
        from .decider import DeciderContext, attach

        root = os.environ.get("SUFFIX_PPLX_DECIDER_DIR") or getattr(aeng.engine.cfg, "weights", None)
        ctx = None
        if root and os.path.exists(os.path.join(root, "decision_config.json")):
            ctx = DeciderContext.load(root, aeng.engine.model, {model_name})
        attach(app, aeng, tokenizer, ctx, aeng.engine.max_model_len)

    return app
