"""Expert parallelism without a cluster: 2 CPU ranks over gloo reproduce EP=1.

Each rank holds half of the routed experts, computes only its (token, expert)
pairs and the partial outputs are all-reduced; greedy generations (with
speculative decoding) must equal the single-rank model's for the Qwen3-Next
hybrid and the DeepSeek/Kimi MLA MoE architectures.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _cfg(name, ep):
    from vllm_suffix_hybrid_b200.engine.config import (CacheConfig, EngineConfig, ParallelConfig, SpecConfig,
                                                       kimi_k2_config, qwen3_next_config, shrink)

    if name == "qwen3_next":
        m = shrink(qwen3_next_config(), layers=4, hidden=128, vocab=512)
    else:
        m = shrink(kimi_k2_config(), layers=3, hidden=128, vocab=512)
        m.weight_format = "bf16"
    m.dtype = "float32"
    return EngineConfig(model=m, spec=SpecConfig(method="hybrid", k=3), parallel=ParallelConfig(ep=ep),
                        cache=CacheConfig(max_model_len=256), max_num_seqs=3, device="cpu", cuda_graphs=False)


def _prompts():
    rng = np.random.default_rng(9)
    return [rng.integers(0, 512, n) for n in (21, 13, 30)]


def _worker(rank, world, port, name, out_q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    torch.set_num_threads(1)
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
    from vllm_suffix_hybrid_b200.parallel import state

    state.init(ep=world, backend="gloo", timeout_s=60)
    try:
        eng = LLMEngine(_cfg(name, world))
        assert eng.model.layers[-1].__dict__.get("moe", getattr(eng.model.layers[-1], "ffn", None)).E_local == \
            eng.cfg.model.num_experts // world
        out_q.put((rank, eng.generate(_prompts(), max_new_tokens=10)))
    finally:
        state.shutdown()


@pytest.mark.parametrize("name", ["qwen3_next", "kimi_k2"])
def test_ep2_matches_ep1(name):
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
    from vllm_suffix_hybrid_b200.parallel import state

    state._STATE = state.ParallelState()
    threads = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        base = LLMEngine(_cfg(name, 1)).generate(_prompts(), max_new_tokens=10)
    finally:
        torch.set_num_threads(threads)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, name, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0] == results[1] == base
