"""Custom-class proposer (Engine): identity, ingestion, arbitration, bounds."""
import json
import os
import tempfile
from types import SimpleNamespace

import numpy as np
import pytest

from vllm_suffix_hybrid_b200.proposer import HybridProposer


def cfg(max_len=256, k=4):
    return SimpleNamespace(speculative_config=SimpleNamespace(num_speculative_tokens=k),
                           model_config=SimpleNamespace(max_model_len=max_len))


@pytest.fixture(autouse=True)
def env():
    saved = {k: v for k, v in os.environ.items() if k.startswith("SUFFIX_HYBRID")}
    for k in list(saved):
        del os.environ[k]
    os.environ.update({"SUFFIX_HYBRID_INDEX_N": "2", "SUFFIX_HYBRID_NGRAM_MIN": "2", "SUFFIX_HYBRID_NGRAM_MAX": "4"})
    yield
    for k in [k for k in os.environ if k.startswith("SUFFIX_HYBRID")]:
        del os.environ[k]
    os.environ.update(saved)


def call(p, rows, sampled=None, dtype=np.int32):
    if sampled is None:
        sampled = [[r[-1]] if r else [] for r in rows]
    buf = np.full((len(rows), 256), -999, dtype=dtype)
    for i, r in enumerate(rows):
        buf[i, :len(r)] = r
    return p.propose(sampled, np.array([len(r) for r in rows], dtype=dtype), buf, slot_mappings=None)


def test_ngram_from_own_history():
    p = HybridProposer(cfg())
    assert call(p, [[1, 2, 3, 4, 1, 2]]) == [[3, 4, 1, 2]]
    assert p.get_stats()["ngram_proposals"] == 1


def test_sampled_tokens_are_not_appended_twice():
    os.environ["SUFFIX_HYBRID_USE_NGRAM"] = "0"
    p = HybridProposer(cfg())
    call(p, [[1, 2, 3, 4]], [[3, 4]])
    call(p, [[7, 8, 9, 10]])
    assert p.suffix_cache.speculate([1, 2], 4)[0] == [3, 4]
    assert p.suffix_cache.stats()["cached_tokens"] == 4
    assert call(p, [[1, 2, 3]]) == [[4]]


def test_equal_counts_are_not_identity():
    p = HybridProposer(cfg())
    call(p, [[1, 2, 3]])
    call(p, [[8, 9, 10, 11]])
    call(p, [])
    assert p.suffix_cache.stats()["cached_tokens"] == 7
    assert p.suffix_cache.speculate([2, 3], 4)[0] == []


def test_reordered_rows_keep_identity_and_grow():
    p = HybridProposer(cfg())
    call(p, [[1, 2, 3], [8, 9, 10]])
    call(p, [[8, 9, 10, 11], [1, 2, 3, 4]])
    assert p.suffix_cache.stats()["num_sequences"] == 0
    call(p, [[1, 2, 3, 4, 5]])
    assert p.suffix_cache.stats()["cached_tokens"] == 4
    call(p, [])
    assert p.suffix_cache.stats()["cached_tokens"] == 9
    assert p.get_stats()["active_requests"] == 0


def test_empty_sampled_and_context_limit():
    p = HybridProposer(cfg(max_len=7))
    row = [1, 2, 3, 4, 1, 2]
    assert call(p, [row], [[]]) == [[]]
    assert call(p, [row]) == [[3]]
    assert call(p, [row + [3]]) == [[]]


def test_int64_and_strided_buffers():
    p = HybridProposer(cfg())
    assert call(p, [[1, 2, 3, 4, 1, 2]], dtype=np.int64) == [[3, 4, 1, 2]]
    a = np.array([[1, 99, 2, 99, 3, 99, 4, 99, 1, 99, 2, 99]], dtype=np.int32)[:, ::2]
    assert p.propose([[2]], np.array([6], dtype=np.int32), a) == [[3, 4, 1, 2]]


def test_invalid_bounds_fail_before_mutation():
    p = HybridProposer(cfg())
    for counts in ([-1], [5], []):
        with pytest.raises(ValueError):
            p.propose([[1]], np.array(counts, dtype=np.int32), np.zeros((1, 4), dtype=np.int32))
    assert p.get_stats()["active_requests"] == 0
    with pytest.raises(ValueError):
        p.propose([[1]], [1], np.zeros((1, 4), dtype=np.int32))  # not a NumPy array


def test_metrics_do_not_claim_acceptance():
    p = HybridProposer(cfg())
    call(p, [[1, 2, 3, 4, 1, 2]])
    st = p.get_stats()
    assert st["accepted"] is None and st["acceptance_rate"] is None
    assert st["native_time_ns"] > 0
    assert st["total_proposer_time_ns"] >= st["native_time_ns"]
    assert "native" in st["version"]


def test_stats_file_and_log_line(caplog):
    with tempfile.TemporaryDirectory() as d:
        os.environ["SUFFIX_HYBRID_STATS_FILE"] = d + "/stats.jsonl"
        os.environ["SUFFIX_HYBRID_STATS_INTERVAL"] = "1"
        os.environ["SUFFIX_HYBRID_LOG_INTERVAL"] = "1"
        p = HybridProposer(cfg())
        with caplog.at_level("INFO", logger="suffix_hybrid"):
            call(p, [[1, 2, 3]])
        rec = json.loads(open(d + "/stats.jsonl").readline())
        assert "native_time_ns" in rec
        assert any("suffix_hybrid" in r.getMessage() for r in caplog.records)


def test_variable_growth_uses_authoritative_rows():
    p = HybridProposer(cfg())
    call(p, [[1, 2, 3]], [[3]])
    call(p, [[1, 2, 3, 4, 5, 6]], [[4, 5, 6]])
    call(p, [[1, 2, 3, 4, 5, 6, 7]], [[7]])
    assert p.get_stats()["active_context_tokens"] == 7
    call(p, [])
    assert p.suffix_cache.stats()["cached_tokens"] == 7


def test_padded_buffers_are_never_listified():
    class NoList(np.ndarray):
        def tolist(self):
            raise AssertionError("converted to list")

    p = HybridProposer(cfg())
    tokens = np.zeros((8, 200_000), dtype=np.int32).view(NoList)
    tokens[0, :6] = [1, 2, 3, 4, 1, 2]
    counts = np.array([6] + [-999] * 7, dtype=np.int32).view(NoList)
    assert p.propose([[2]], counts, tokens) == [[3, 4, 1, 2]]


def test_suffix_confidence_beats_ngram():
    p = HybridProposer(cfg())
    p.suffix_cache.add_sequence([3, 4, 1, 2, 91, 92, 93, 94])
    assert call(p, [[1, 2, 3, 4, 1, 2]]) == [[91, 92, 93, 94]]
    assert p.get_stats()["suffix_proposals"] == 1


def test_compat_alias_package():
    from suffix_hybrid._native import Engine, VERSION  # noqa: F401
    from suffix_hybrid.hybrid_proposer import HybridProposer as Alias
    from suffix_hybrid.suffix_cache import SuffixCache  # noqa: F401
    assert Alias is HybridProposer
