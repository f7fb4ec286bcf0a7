"""Tensor parallelism without a cluster: 2 CPU ranks over gloo reproduce TP=1.

Checks the column/row sharding of fused QKV and gate|up weights, the
all-reduce placement, and the vocab-parallel greedy argmax (no logits
gather) end to end through the engine.
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


def _cfg(method):
    from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig, llama3_8b_config, shrink

    m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=512)
    m.dtype = "float32"
    return EngineConfig(model=m, spec=SpecConfig(method=method, k=3), cache=CacheConfig(max_model_len=256),
                        max_num_seqs=3, device="cpu", cuda_graphs=False)


def _prompts():
    rng = np.random.default_rng(5)
    return [rng.integers(0, 512, n) for n in (30, 17, 41)]


def _worker(rank, world, port, method, out_q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
    from vllm_suffix_hybrid_b200.parallel import state

    torch.set_num_threads(1)  # fixed CPU reduction order in every process
    state.init(tp=world, backend="gloo", timeout_s=60)
    try:
        eng = LLMEngine(_cfg(method))
        out_q.put((rank, eng.generate(_prompts(), max_new_tokens=12)))
    finally:
        state.shutdown()


@pytest.mark.parametrize("method", ["hybrid", "none"])
def test_tp2_matches_tp1(method):
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
    from vllm_suffix_hybrid_b200.parallel import state

    state._STATE = state.ParallelState()
    threads = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        base = LLMEngine(_cfg(method)).generate(_prompts(), max_new_tokens=12)
    finally:
        torch.set_num_threads(threads)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, method, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0] == results[1] == base
