"""Online draft-head tuning on CPU: the zero-initialised adapter is an exact no-op for serving, the
differentiable replay reproduces the serving draft chain, training lowers the loss, the gate promotes
in place, rollback zeroes the live adapter, and the TP autograd collectives are consistent over gloo."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig, llama3_8b_config, shrink
from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
from vllm_suffix_hybrid_b200.tune import replay


def _cfg(method="hybrid", k=4):
    m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=512)
    m.dtype = "float32"
    return EngineConfig(model=m, spec=SpecConfig(method=method, k=k), cache=CacheConfig(max_model_len=512),
                        max_num_seqs=2, device="cpu", cuda_graphs=False)


@pytest.fixture
def tune_env(monkeypatch, tmp_path):
    monkeypatch.setenv("SUFFIX_MTP_TUNE", "1")
    monkeypatch.setenv("SUFFIX_MTP_TUNE_RATE", "1.0")
    monkeypatch.setenv("SUFFIX_MTP_TUNE_HELDOUT_PCT", "30")
    monkeypatch.setenv("SUFFIX_MTP_TUNE_MIN_TRAIN_WINDOWS", "2")
    monkeypatch.setenv("SUFFIX_MTP_TUNE_MIN_EVAL_WINDOWS", "1")
    monkeypatch.setenv("SUFFIX_MTP_TUNE_MIN_ANCHORS", "10")
    monkeypatch.setenv("SUFFIX_MTP_TUNE_ROLLBACK_FILE", str(tmp_path / "rollback"))
    return tmp_path


def test_zero_adapter_is_a_no_op(tune_env):
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 512, 20) for _ in range(3)]
    os.environ.pop("SUFFIX_MTP_TUNE")
    base = LLMEngine(_cfg()).generate(prompts, max_new_tokens=12)
    os.environ["SUFFIX_MTP_TUNE"] = "1"
    eng = LLMEngine(_cfg())
    assert eng.tuner is not None and all(l.lora is not None for l in eng.tuner.lin.values())
    assert eng.generate(prompts, max_new_tokens=12) == base
    assert eng.tuner.stats["captured"] == 3


def test_replay_matches_the_serving_draft_chain(tune_env):
    eng = LLMEngine(_cfg("native", k=4))
    prompt = np.random.default_rng(1).integers(0, 512, 30)
    first, natives = eng.runner.prefill([prompt], [eng.pool.allocate(2)], [0])
    seq = torch.from_numpy(np.concatenate([prompt, [int(first[0])]]))
    feats = eng.features(seq.numpy())
    anchor = torch.tensor([len(prompt) - 1])
    _, toks = replay.chain_accept(eng.draft, None, seq, feats, anchor, 4, return_tokens=True)
    assert toks[0].tolist() == natives[0][:4].tolist()


def test_training_gate_promotion_and_rollback(tune_env, monkeypatch):
    monkeypatch.setenv("SUFFIX_MTP_TUNE_LR", "3e-3")
    monkeypatch.setenv("SUFFIX_MTP_TUNE_ACCUM", "2")
    monkeypatch.setenv("SUFFIX_MTP_TUNE_STEP_MS", "1")  # one sequence per micro-step: load-independent
    monkeypatch.setenv("SUFFIX_MTP_TUNE_EVAL_EVERY", "100000")
    eng = LLMEngine(_cfg())
    tuner = eng.tuner
    rng = np.random.default_rng(3)
    motif = rng.integers(0, 512, 12)
    for i in range(10):  # repetitive traffic the random head can learn
        seq = np.concatenate([rng.integers(0, 512, 6), np.tile(motif, 6)])
        tuner.capture(f"req-{i}", seq)
    assert len(tuner.train) >= 2 and len(tuner.heldout) >= 1
    first = None
    while tuner.stats["opt_steps"] < 60:
        tuner.micro_step()
        first = first if first is not None else tuner.stats["last_loss"]
    assert tuner.stats["last_loss"] < first
    live, cand, anchors, _ = tuner.evaluate()
    assert anchors > 0 and cand > live
    tuner.promote()
    for n, (a, b) in tuner.live.items():
        assert torch.equal(b, tuner.cand[n][1].detach().to(b.dtype))
    assert any(float(b.abs().sum()) > 0 for _, b in tuner.live.values())
    (tune_env / "rollback").write_text("")
    tuner.micro_step()
    assert all(float(b.abs().sum()) == 0 for _, b in tuner.live.values()) and not tuner.promote_ok


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _collectives_worker(rank, port, q):
    import torch.distributed as dist

    from vllm_suffix_hybrid_b200.parallel import state
    from vllm_suffix_hybrid_b200.tune import collectives as C

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    st = state.ParallelState()
    st.tp, st.tp_rank, st.world, st.rank, st.group, st.cpu_group = 2, rank, 2, rank, dist.group.WORLD, dist.group.WORLD
    state._STATE = st
    torch.manual_seed(0)
    w = torch.randn(6, 4)  # full column-parallel weight, rows split over the ranks
    x = torch.randn(3, 4, requires_grad=True)
    y = C.gather_from_tp(C.copy_to_tp(x) @ w[rank * 3:(rank + 1) * 3].t())
    y.pow(2).sum().backward()
    xf = x.detach().clone().requires_grad_(True)
    (xf @ w.t()).pow(2).sum().backward()
    r = C.reduce_from_tp(torch.full((2,), float(rank + 1)))
    q.put((rank, torch.allclose(x.grad, xf.grad, atol=1e-5), torch.allclose(y, xf.detach() @ w.t(), atol=1e-5),
           r.tolist()))
    dist.destroy_process_group()


def test_tp_autograd_collectives_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_collectives_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = [q.get(timeout=120) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, grad_ok, fwd_ok, red in out:
        assert grad_ok and fwd_ok and red == [3.0, 3.0]
