"""In-place SFT routes (SUFFIX_SFT=1 with SUFFIX_SFT_TOKEN set; see tune/sft.py).

  POST /v1/sft/train   {"examples": [{"messages": [...]} | {"prompt": str, "completion": str}], "steps": 1,
                        "batch_size": 1, "learning_rate": 1e-4, "weight_decay": 0.0, "run_id": opt., "wait": true}
  POST /v1/sft/load    {"run_id": "<saved run>" | "base"}
  GET  /v1/sft/status
train and load need the header X-SFT-Token: <SUFFIX_SFT_TOKEN> (without a token the routes refuse, so a
server can not be retrained by every client).  Chat examples train on the final assistant message (the
prompt is the history rendered with the generation prompt, as serving renders it); raw examples train on
the completion followed by EOS.  Reference: suffix_hybrid/sft/api.py:1-40.
"""
import asyncio
import os

from fastapi import Request
from fastapi.responses import JSONResponse


def _tokenize(tokenizer, ex):
    eos = getattr(tokenizer, "eos_token_id", None)
    tail = [eos] if eos is not None else []
    if "messages" in ex:
        msgs = ex["messages"]
        if not isinstance(msgs, list) or not msgs or msgs[-1].get("role") != "assistant":
            raise ValueError("chat examples end with an assistant message")
        prompt = list(tokenizer.apply_chat_template(msgs[:-1]))
        target = list(tokenizer.encode(str(msgs[-1].get("content", "")))) + tail
    elif "prompt" in ex and "completion" in ex:
        prompt = list(tokenizer.encode(str(ex["prompt"])))
        target = list(tokenizer.encode(str(ex["completion"]))) + tail
    else:
        raise ValueError("an example is {\"messages\": [...]} or {\"prompt\": ..., \"completion\": ...}")
    if not prompt:
        raise ValueError("an example needs a non-empty prompt")
    return prompt, target


def attach(app, aeng, tokenizer) -> None:
    token = os.environ.get("SUFFIX_SFT_TOKEN", "")

    def denied(request: Request):
        if not token:
            return JSONResponse({"error": "SFT routes need SUFFIX_SFT_TOKEN on the server"}, status_code=403)
        if request.headers.get("x-sft-token") != token:
            return JSONResponse({"error": "bad or missing X-SFT-Token"}, status_code=401)
        return None

    @app.get("/v1/sft/status")
    async def sft_status():
        sft = aeng.engine.sft
        return {"enabled": sft is not None, **(dict(sft.status) if sft is not None else {})}

    @app.post("/v1/sft/train")
    async def sft_train(request: Request):
        if (err := denied(request)) is not None:
            return err
        try:
            body = await request.json()
            examples = [_tokenize(tokenizer, ex) for ex in body.get("examples") or []]
            kw = dict(examples=examples, steps=int(body.get("steps", 1)), batch_size=int(body.get("batch_size", 1)),
                      learning_rate=float(body.get("learning_rate", 1e-4)),
                      weight_decay=float(body.get("weight_decay", 0.0)), run_id=body.get("run_id"))
        except (ValueError, TypeError, AttributeError) as ex:
            return JSONResponse({"error": str(ex)}, status_code=400)
        try:
            run_id = await aeng.sft_call("sft_begin", kw)
        except (ValueError, RuntimeError) as ex:
            return JSONResponse({"error": str(ex)}, status_code=409)
        if not body.get("wait", True):
            return JSONResponse({"run_id": run_id, "state": "training"}, status_code=202)
        sft = aeng.engine.sft
        while sft.run is not None:
            await asyncio.sleep(0.05)
        st = dict(sft.status)
        return JSONResponse(st, status_code=200 if st.get("state") == "idle" else 500)

    @app.post("/v1/sft/load")
    async def sft_load(request: Request):
        if (err := denied(request)) is not None:
            return err
        try:
            body = await request.json()
            await aeng.sft_call("sft_load", str(body["run_id"]))
        except (KeyError, ValueError, TypeError, FileNotFoundError, RuntimeError) as ex:
            return JSONResponse({"error": str(ex)}, status_code=400)
        return dict(aeng.engine.sft.status)
