"""SUFFIX_HYBRID_SPLIT=diverge: counterfactual arbitration at the first disagreement."""
import pytest

from vllm_suffix_hybrid_b200._native import HybridMixer

CTX = list(range(1, 9))


@pytest.fixture
def diverge(monkeypatch):
    monkeypatch.setenv("SUFFIX_HYBRID_SPLIT", "diverge")
    monkeypatch.setenv("SUFFIX_HYBRID_INDEX_N", "2")


def mixer():
    m = HybridMixer(5, 1024)
    m.suffix_cache.add_sequence(list(range(1, 200)))
    return m


def test_untrained_bucket_keeps_native(diverge):
    m = mixer()
    assert m.mix(["a"], [CTX], [[9, 10, 99, 98, 97]], None) == [[9, 10, 99, 98, 97]]
    assert m.last_native_counts() == [5]
    assert m.get_stats()["split_mode"] == "diverge"


def test_suffix_right_trains_trust_then_overlays(diverge):
    m = mixer()
    m.mix(["a"], [CTX], [[9, 10, 99, 98, 97]], None)
    got = m.mix(["a"], [CTX + [9, 10, 11]], [[12, 13, 77, 76, 75]], [2])
    assert m.get_stats()["div_observed"] == 1
    assert got == [[12, 13, 14, 15, 16]] and m.last_native_counts() == [2]


def test_native_right_keeps_native(diverge):
    m = mixer()
    m.mix(["a"], [CTX], [[9, 10, 99, 98, 97]], None)
    assert m.mix(["a"], [CTX + [9, 10, 99]], [[5, 6, 7, 8, 9]], [2]) == [[5, 6, 7, 8, 9]]
    assert max(m.get_stats()["div_trust"]) <= 0.5


def test_unreached_divergence_is_censored(diverge):
    m = mixer()
    m.mix(["a"], [CTX], [[9, 10, 99, 98, 97]], None)
    m.mix(["a"], [CTX + [9, 55]], [[1, 2, 3, 4, 5]], [1])
    assert m.get_stats()["div_observed"] == 0


def test_in_request_ngram_candidate(diverge, monkeypatch):
    monkeypatch.setenv("SUFFIX_HYBRID_SELF_NGRAM_MIN", "3")
    m = HybridMixer(5, 1024)
    ctx = [7, 8, 9, 40, 41, 42, 43, 44, 3, 3, 7, 8, 9]
    m.mix(["a"], [ctx], [[40, 41, 90, 91, 92]], None)
    assert m.get_stats()["self_hits"] == 1
    m.mix(["a"], [ctx + [40, 41, 42]], [[43, 44, 1, 1, 1]], [2])
    assert m.get_stats()["div_observed"] == 1
