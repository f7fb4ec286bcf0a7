"""Decision endpoint (SUFFIX_PPLX_DECIDER=1): POST /v1/systemone classifies a state against questions.

A decision checkpoint directory (SUFFIX_PPLX_DECIDER_DIR, else the served weights directory) holds
`decision_config.json`: 255 answer `codes` with their single-token `token_ids`, a positive `temperature`
and an optional `prompt` family ("d3"; absent = pplx).  The readout is `readout.safetensors` ("weight"
[255, H]) when present, else the served model's LM-head rows of the code tokens.  Per question the native
helpers render the prompt (decider_prepare), the engine scores the chat-templated prompt at its last
position against the readout rows (LLMEngine.readout), and decider_answer reduces the logits to the
answer.  Reference: suffix_hybrid_decider_ep.py:24-112 (route, flow, error mapping),
suffix_hybrid/decider_contract.py:14-50 (checkpoint contract).
Deviations: the backbone is the served causal model (the reference's decision checkpoints use
non-causal full attention over the prompt); text only (image / video inputs are refused); one rank.
"""
from __future__ import annotations

import json
import math
import os
from typing import Optional

import torch
from fastapi import Request
from fastapi.responses import JSONResponse

PROFILES = {None: "pplx", "d3": "d3"}


class DeciderContext:
    def __init__(self, codes, token_ids, temperature: float, profile: str, rows: torch.Tensor, names):
        self.codes, self.token_ids = list(codes), list(token_ids)
        self.temperature, self.profile = float(temperature), profile
        self.rows = rows
        self.names = set(names)

    @classmethod
    def load(cls, root: str, model, names) -> "DeciderContext":
        cfg_path = os.path.join(root, "decision_config.json")
        with open(cfg_path) as fh:
            saved = json.load(fh)
        codes, ids = saved.get("codes"), saved.get("token_ids")
        if (not isinstance(codes, list) or len(codes) != 255 or len(set(codes)) != 255
                or any(not isinstance(c, str) or not c for c in codes)
                or not isinstance(ids, list) or len(ids) != 255 or len(set(ids)) != 255
                or any(type(t) is not int or t < 0 for t in ids)):
            raise ValueError("decision checkpoint must declare 255 unique codes / token ids")
        t = saved.get("temperature")
        if type(t) not in (int, float) or not math.isfinite(t) or t <= 0:
            raise ValueError("decision checkpoint temperature must be finite and positive")
        if saved.get("prompt") not in PROFILES:
            raise ValueError("unknown decision prompt family")
        ro = os.path.join(root, "readout.safetensors")
        if os.path.exists(ro):
            from safetensors.torch import load_file

            rows = load_file(ro)["weight"]
        else:
            head = getattr(model, "lm_head", None)
            w = getattr(head, "weight", None)
            if w is None or max(ids) >= w.shape[0]:
                raise ValueError("no readout.safetensors and the LM head can not read out the code tokens")
            rows = w.index_select(0, torch.tensor(ids, device=w.device))
        return cls(codes, ids, t, PROFILES[saved.get("prompt")], rows.detach().clone(), names)


def _text_messages(messages):
    """Chat messages with list content flattened to text (for tokenizers without multimodal templates)."""
    out = []
    for m in messages:
        c = m.get("content")
        if isinstance(c, list):
            c = "".join(p.get("text", "") for p in c if isinstance(p, dict))
        out.append({"role": m.get("role", "user"), "content": c})
    return out


def attach(app, aeng, tokenizer, ctx: Optional[DeciderContext], max_model_len: int) -> None:
    from .. import _native

    @app.post("/v1/systemone")
    async def systemone(request: Request):
        if ctx is None:
            return JSONResponse({"error": "no decision checkpoint configured"}, status_code=404)
        try:
            body = await request.json()
            if isinstance(body, dict) and body.get("model") not in ctx.names:
                return JSONResponse({"error": "Unknown decision model"}, status_code=404)
            body_json = json.dumps(body, ensure_ascii=False)
            prepared = json.loads(_native.decider_prepare(body_json, json.dumps(ctx.codes), ctx.profile))
            if body.get("images") or body.get("videos"):
                raise ValueError("this server's decision endpoint supports text only")
            prompts = []
            for row in prepared["rows"]:
                ids = list(tokenizer.apply_chat_template(_text_messages(row["messages"])))
                if not ids or len(ids) > max_model_len:
                    raise ValueError("decision input must fit model limit without truncation")
                prompts.append(ids)
        except (ValueError, TypeError, KeyError) as error:
            return JSONResponse({"error": str(error)}, status_code=400)
        logits = [await aeng.readout(ids, ctx.rows) for ids in prompts]
        resp = json.loads(_native.decider_answer(body_json, json.dumps(logits), ctx.temperature, ctx.profile))
        resp["usage"]["input_tokens"] = sum(len(p) for p in prompts)
        return JSONResponse(resp)
