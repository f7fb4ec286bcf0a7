"""HTTP serving on CPU: OpenAI-style routes over AsyncEngine, greedy outputs equal LLMEngine's,
streaming equals non-streaming, warm start, metrics; TP=2 lockstep over gloo."""
import asyncio
import json
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _cfg(method="hybrid"):
    from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig, llama3_8b_config, shrink

    m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=512)
    m.dtype = "float32"
    return EngineConfig(model=m, spec=SpecConfig(method=method, k=3), cache=CacheConfig(max_model_len=256),
                        max_num_seqs=3, device="cpu", cuda_graphs=False)


@pytest.fixture(scope="module")
def server():
    from fastapi.testclient import TestClient

    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
    from vllm_suffix_hybrid_b200.parallel import state
    from vllm_suffix_hybrid_b200.serve import AsyncEngine, ByteTokenizer
    from vllm_suffix_hybrid_b200.serve.api_server import build_app

    state._STATE = state.ParallelState()
    os.environ["SUFFIX_HYBRID_WARMSTART"] = "1"
    aeng = AsyncEngine(LLMEngine(_cfg()))
    aeng.start()
    app = build_app(aeng, ByteTokenizer(), "toy")
    with TestClient(app) as client:
        yield client, aeng
    aeng.shutdown()
    os.environ.pop("SUFFIX_HYBRID_WARMSTART", None)


def _plain(prompt, n):
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine

    return LLMEngine(_cfg("none")).generate([prompt], n)[0]


def test_routes_and_greedy_equivalence(server):
    client, _ = server
    assert client.get("/health").json()["status"] == "ok"
    assert client.get("/v1/models").json()["data"][0]["id"] == "toy"
    prompt = list(range(20, 45))
    r = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 10, "ignore_eos": True})
    assert r.status_code == 200, r.text
    body = r.json()
    assert body["choices"][0]["token_ids"] == _plain(prompt, 10)
    assert body["usage"]["completion_tokens"] == 10 and body["choices"][0]["finish_reason"] == "length"


def test_streaming_matches_non_streaming(server):
    client, _ = server
    prompt = list(range(60, 90))
    whole = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 9, "ignore_eos": True}).json()
    toks, reasons = [], []
    with client.stream("POST", "/v1/completions",
                       json={"prompt": prompt, "max_tokens": 9, "stream": True, "ignore_eos": True}) as r:
        for line in r.iter_lines():
            if not line.startswith("data: ") or line == "data: [DONE]":
                continue
            ch = json.loads(line[6:])["choices"][0]
            toks += ch["token_ids"]
            reasons.append(ch["finish_reason"])
    assert toks == whole["choices"][0]["token_ids"] and reasons[-1] == "length"


def test_chat_text_prompt_stop_and_errors(server):
    client, _ = server
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4})
    assert r.status_code == 200 and r.json()["object"] == "chat.completion"
    assert client.post("/v1/completions", json={"prompt": "abc", "temperature": 0.7}).status_code == 400
    assert client.post("/v1/chat/completions", json={"messages": []}).status_code == 400
    prompt = list(range(100, 130))
    ref = _plain(prompt, 8)
    r = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 8, "stop_token_ids": [ref[2]],
                                             "ignore_eos": True}).json()
    cut = ref.index(ref[2]) + 1
    assert r["choices"][0]["token_ids"] == ref[:cut] and r["choices"][0]["finish_reason"] == "stop"


def test_concurrent_requests(server):
    client, _ = server
    import concurrent.futures as cf

    prompts = [list(range(s, s + 15)) for s in (5, 200, 300, 400)]
    with cf.ThreadPoolExecutor(4) as ex:
        outs = list(ex.map(lambda p: client.post("/v1/completions", json={"prompt": p, "max_tokens": 6,
                                                                             "ignore_eos": True}).json(), prompts))
    for p, o in zip(prompts, outs):
        assert o["choices"][0]["token_ids"] == _plain(p, 6)


def test_warm_start_and_metrics(server):
    client, aeng = server
    r = client.post("/debug/warm-start", json={"sequences": [[1, 2, 3, 4, 5, 6, 7, 8, 9] * 3, [7, 7, 7, 7, 7] * 4]})
    assert r.json() == {"ingested": 2}
    assert client.post("/debug/warm-start", json={"sequences": "x"}).status_code == 400
    text = client.get("/metrics").text
    assert "suffix_hybrid_requests_finished" in text and "suffix_hybrid_warm_start_sequences_total 2" in text
    st = client.get("/v1/spec_stats").json()
    assert st["requests_finished"] >= 1 and "proposer" in st


def test_corpus_save_route(server, tmp_path):
    from vllm_suffix_hybrid_b200 import _native

    client, aeng = server
    client.post("/debug/warm-start", json={"sequences": [[3, 1, 4, 1, 5, 9, 2, 6] * 4]})
    path = str(tmp_path / "corpus.bin")
    r = client.post("/debug/corpus-save", json={"path": path})
    n = aeng.engine.proposer.suffix_cache.stats()["num_sequences"]
    assert r.status_code == 200 and r.json() == {"saved": n, "path": path} and n >= 1
    assert _native.SuffixCache().load(path) == n
    assert client.post("/debug/corpus-save", json={}).status_code == 400  # no path and no default file
    assert client.post("/debug/corpus-save", json={"path": str(tmp_path / "no" / "dir.bin")}).status_code == 409


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _tp_worker(rank, world, port, out_q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    torch.set_num_threads(1)
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
    from vllm_suffix_hybrid_b200.parallel import state
    from vllm_suffix_hybrid_b200.serve import AsyncEngine

    st = state.init(tp=world, backend="gloo", timeout_s=60)
    try:
        aeng = AsyncEngine(LLMEngine(_cfg()), st.rank, st.world, st.cpu_group)
        if rank != 0:
            aeng.worker_loop()
            return
        aeng.start()

        async def one(p):
            toks = []
            async for new, fin, _ in aeng.generate(p, 8):
                toks += new
            return toks

        async def main():
            return await asyncio.gather(*(one(list(range(s, s + 20))) for s in (3, 50, 99)))

        out_q.put(asyncio.run(main()))
        aeng.shutdown()
    finally:
        state.shutdown()


def test_tp2_lockstep_serving():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    threads = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        from vllm_suffix_hybrid_b200.parallel import state

        state._STATE = state.ParallelState()
        want = [_plain(list(range(s, s + 20)), 8) for s in (3, 50, 99)]
    finally:
        torch.set_num_threads(threads)
    assert got == want


def test_step_profiler_windows(tmp_path, monkeypatch):
    """SUFFIX_HYBRID_STEP_PROFILE writes a trace and a kernel/op summary per batch bucket."""
    monkeypatch.setenv("SUFFIX_HYBRID_STEP_PROFILE", str(tmp_path))
    monkeypatch.setenv("SUFFIX_HYBRID_STEP_PROFILE_SKIP", "1")
    monkeypatch.setenv("SUFFIX_HYBRID_STEP_PROFILE_STEPS", "2")
    monkeypatch.setenv("SUFFIX_HYBRID_STEP_PROFILE_BUCKETS", "2,8")
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
    from vllm_suffix_hybrid_b200.parallel import state

    state._STATE = state.ParallelState()
    eng = LLMEngine(_cfg("hybrid"))
    eng.generate([list(range(5, 25)), list(range(40, 60))], 8)
    files = sorted(os.listdir(tmp_path))
    assert "step_b2_r0.txt" in files and "step_b2_r0.json" in files, files
    assert open(tmp_path / "step_b2_r0.txt").read().startswith("# 2 decode steps")
