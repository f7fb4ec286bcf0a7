"""In-place SFT on CPU: zero adapters change nothing; the training replay reproduces the served greedy
tokens; training on a prompt / completion pair makes the SERVED engine generate the completion; runs
checkpoint, restore at the next start and roll back to base; the HTTP routes need the token."""
import numpy as np
import pytest
import torch

from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig, llama3_8b_config, shrink
from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
from vllm_suffix_hybrid_b200.tune import replay


def _cfg(method="none"):
    m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=512)
    m.dtype = "float32"
    return EngineConfig(model=m, spec=SpecConfig(method=method, k=3), cache=CacheConfig(max_model_len=256),
                        max_num_seqs=2, device="cpu", cuda_graphs=False)


@pytest.fixture
def sft_env(monkeypatch, tmp_path):
    monkeypatch.setenv("SUFFIX_SFT", "1")
    monkeypatch.setenv("SUFFIX_SFT_DIR", str(tmp_path / "sft"))
    return tmp_path


PROMPT = np.arange(40, 60)
COMPLETION = [7, 100, 42, 300, 9, 77, 250, 13]


def test_zero_adapters_and_replay_parity(sft_env):
    import os

    os.environ.pop("SUFFIX_SFT")
    base = LLMEngine(_cfg("hybrid")).generate([PROMPT], max_new_tokens=10)[0]
    os.environ["SUFFIX_SFT"] = "1"
    eng = LLMEngine(_cfg("hybrid"))
    assert eng.sft is not None and len(eng.sft.live) == 8  # 2 layers x qkv / o / gate_up / down
    assert eng.generate([PROMPT], max_new_tokens=10)[0] == base
    seq = torch.tensor(list(PROMPT) + base)
    with torch.no_grad():
        logits = replay.target_logits(eng.model, None, seq[:-1])
    assert logits[len(PROMPT) - 1:].argmax(-1).tolist() == base


def test_training_changes_serving_in_place_and_checkpoints(sft_env):
    eng = LLMEngine(_cfg())
    base = eng.generate([PROMPT], max_new_tokens=len(COMPLETION))[0]
    assert base != COMPLETION
    run = eng.sft.begin([(list(PROMPT), COMPLETION)], steps=120, learning_rate=3e-3, run_id="memo")
    while eng.sft.run is not None:
        eng.sft.micro()
    assert eng.sft.status["state"] == "idle" and eng.sft.status["run_id"] == run
    assert eng.generate([PROMPT], max_new_tokens=len(COMPLETION))[0] == COMPLETION
    fresh = LLMEngine(_cfg())  # restores latest.json at start
    assert fresh.sft.status["run_id"] == "memo"
    assert fresh.generate([PROMPT], max_new_tokens=len(COMPLETION))[0] == COMPLETION
    fresh.sft.load("base")
    assert fresh.generate([PROMPT], max_new_tokens=len(COMPLETION))[0] == base
    assert LLMEngine(_cfg()).sft.status["run_id"] == "base"


def test_routes_require_the_token(sft_env, monkeypatch):
    from fastapi.testclient import TestClient

    from vllm_suffix_hybrid_b200.parallel import state
    from vllm_suffix_hybrid_b200.serve import AsyncEngine, ByteTokenizer
    from vllm_suffix_hybrid_b200.serve.api_server import build_app

    monkeypatch.setenv("SUFFIX_SFT_TOKEN", "s3cret")
    state._STATE = state.ParallelState()
    aeng = AsyncEngine(LLMEngine(_cfg()))
    aeng.start()
    try:
        with TestClient(build_app(aeng, ByteTokenizer(), "toy")) as c:
            body = {"examples": [{"prompt": "hi", "completion": "yo"}], "steps": 2, "learning_rate": 1e-3}
            assert c.post("/v1/sft/train", json=body).status_code == 401
            r = c.post("/v1/sft/train", json=body, headers={"X-SFT-Token": "s3cret"})
            assert r.status_code == 200, r.text
            assert r.json()["step"] == 2 and r.json()["state"] == "idle"
            assert c.get("/v1/sft/status").json()["enabled"]
            bad = c.post("/v1/sft/train", json={"examples": [{"text": "x"}]}, headers={"X-SFT-Token": "s3cret"})
            assert bad.status_code == 400
            assert c.post("/v1/sft/load", json={"run_id": "base"}, headers={"X-SFT-Token": "s3cret"}).status_code == 200
    finally:
        aeng.shutdown()
