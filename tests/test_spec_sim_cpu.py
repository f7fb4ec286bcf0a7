"""The acceptance simulator drives the real native mixer on scripted workloads."""
import pytest

from vllm_suffix_hybrid_b200.bench.spec_sim import head_draft, simulate, workload


@pytest.mark.parametrize("name", ["fresh", "templated", "echo", "tools"])
def test_workloads_are_seeded_and_shaped(name):
    a = list(workload(name, 10, seed=3))
    b = list(workload(name, 10, seed=3))
    assert a == b and len(a) >= 2
    for prompt, cont, rep in a:
        assert len(cont) == len(rep) == 256 and len(prompt) > 0


def test_head_model_is_wrong_after_its_first_miss():
    import numpy as np

    rng = np.random.default_rng(0)
    truth = list(range(100, 108))
    for _ in range(200):
        d = head_draft(rng, truth, [False] * 8, 8)
        miss = next((i for i, t in enumerate(d) if t != truth[i]), len(d))
        assert all(d[i] != truth[i] for i in range(miss, len(d)))


def test_recurring_requests_gain_from_the_suffix_corpus():
    draft = simulate("templated", "draft", k=5, conc=4, n_req=20)
    diverge = simulate("templated", "diverge", k=5, conc=4, n_req=20)
    again = simulate("templated", "diverge", k=5, conc=4, n_req=20)
    assert diverge["tokens_per_step"] == again["tokens_per_step"]  # deterministic for a seed
    assert diverge["tokens_per_step"] > draft["tokens_per_step"] + 0.5
    assert 1.0 <= draft["tokens_per_step"] <= 6.0
