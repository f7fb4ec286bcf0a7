"""Data-parallel attention + expert parallelism without a cluster: 2 CPU ranks over gloo.

Each rank serves its own requests (different counts, lengths and output budgets, so prefill padding,
decode bucket padding and idle-rank dummy steps all occur); MoE layers gather every rank's tokens, run
the rank's half of the experts and reduce-scatter the outputs.  Each rank's greedy generations (with
speculative decoding) must equal a single process serving the same prompts.
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
    return EngineConfig(model=m, spec=SpecConfig(method="hybrid", k=3), parallel=ParallelConfig(ep=ep, dp=ep),
                        cache=CacheConfig(max_model_len=256), max_num_seqs=3, device="cpu", cuda_graphs=False)


def _work(rank):
    rng = np.random.default_rng(20 + rank)
    if rank == 0:
        return [rng.integers(0, 512, n) for n in (21, 13, 30, 8)], 12
    return [rng.integers(0, 512, 17)], 5


def _worker(rank, world, port, name, out_q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    torch.set_num_threads(1)
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
    from vllm_suffix_hybrid_b200.parallel import state

    state.init(ep=world, dp=world, backend="gloo", timeout_s=60)
    try:
        eng = LLMEngine(_cfg(name, world))
        prompts, new = _work(rank)
        out_q.put((rank, eng.generate(prompts, max_new_tokens=new)))
    finally:
        state.shutdown()


@pytest.mark.parametrize("name", ["qwen3_next", "kimi_k2"])
def test_dp2_attention_matches_single_process(name):
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
    from vllm_suffix_hybrid_b200.parallel import state

    state._STATE = state.ParallelState()
    threads = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        base = {r: LLMEngine(_cfg(name, 1)).generate(*_work(r)) for r in range(2)}
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
    for r in range(2):
        assert results[r] == base[r], (r, results[r], base[r])
