"""/v1/systemone on a CPU engine with a synthetic decision checkpoint (readout = LM-head rows of the code
tokens): answers equal the native reduction of the engine's own readout logits; bad requests map to
404 / 400."""
import json
import os

import pytest
import torch


@pytest.fixture(scope="module")
def client(tmp_path_factory):
    from fastapi.testclient import TestClient

    from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig, llama3_8b_config, shrink
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
    from vllm_suffix_hybrid_b200.parallel import state
    from vllm_suffix_hybrid_b200.serve import AsyncEngine, ByteTokenizer
    from vllm_suffix_hybrid_b200.serve.api_server import build_app

    root = tmp_path_factory.mktemp("decider")
    (root / "decision_config.json").write_text(json.dumps(
        {"codes": [f"C{i}" for i in range(255)], "token_ids": list(range(3, 258)), "temperature": 0.7}))
    state._STATE = state.ParallelState()
    m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=512)
    m.dtype = "float32"
    eng = LLMEngine(EngineConfig(model=m, spec=SpecConfig(method="none"), cache=CacheConfig(max_model_len=1024),
                                 max_num_seqs=2, device="cpu", cuda_graphs=False))
    os.environ["SUFFIX_PPLX_DECIDER"] = "1"
    os.environ["SUFFIX_PPLX_DECIDER_DIR"] = str(root)
    aeng = AsyncEngine(eng)
    aeng.start()
    app = build_app(aeng, ByteTokenizer(), "decider")
    with TestClient(app) as c:
        yield c, eng
    aeng.shutdown()
    os.environ.pop("SUFFIX_PPLX_DECIDER")
    os.environ.pop("SUFFIX_PPLX_DECIDER_DIR")


BODY = {"model": "decider", "state": {"ticket": "refund please"},
        "questions": {"route": {"type": "choice", "criteria": {"billing": None, "tech": "broken app"}},
                      "urgent": {"type": "noul"},
                      "severity": {"type": "score", "criteria": ["low", "mid", "high"]}}}


def test_answers_follow_the_engine_readout(client):
    c, eng = client
    from vllm_suffix_hybrid_b200 import _native
    from vllm_suffix_hybrid_b200.serve import ByteTokenizer
    from vllm_suffix_hybrid_b200.serve.decider import _text_messages

    r = c.post("/v1/systemone", json=BODY)
    assert r.status_code == 200, r.text
    got = r.json()
    assert list(got["answers"]) == ["route", "urgent", "severity"] and got["usage"]["input_tokens"] > 0
    # recompute: same prompts, the engine's readout against the LM-head rows of the code tokens
    body_json = json.dumps(BODY, ensure_ascii=False)
    prep = json.loads(_native.decider_prepare(body_json, json.dumps([f"C{i}" for i in range(255)]), "pplx"))
    rows = eng.model.lm_head.weight.index_select(0, torch.arange(3, 258))
    tok = ByteTokenizer()
    logits = [eng.readout(tok.apply_chat_template(_text_messages(row["messages"])), rows) for row in prep["rows"]]
    want = json.loads(_native.decider_answer(body_json, json.dumps(logits), 0.7, "pplx"))
    assert got["answers"] == want["answers"]
    p = got["answers"]["route"]["probabilities"]
    assert abs(sum(p.values()) - 1.0) < 1e-9


def test_errors(client):
    c, _ = client
    assert c.post("/v1/systemone", json=dict(BODY, model="other")).status_code == 404
    assert c.post("/v1/systemone", json=dict(BODY, images=["data:x"])).status_code == 400
    assert c.post("/v1/systemone", json={"model": "decider", "state": "s", "questions": {}}).status_code == 400
