"""Custom-class HybridProposer: the documented contract, checked as properties.

Contract (module docstring of ``proposer/hybrid_proposer.py``): rows arrive
as authoritative CPU buffers that already hold the sampled tokens; a row
that continues an earlier row keeps its state, a row that leaves the batch
is ingested into the shared suffix corpus, and each draft is at most k
tokens and never runs past max_model_len.
"""
import json
import os
from types import SimpleNamespace

import numpy as np
import pytest

from vllm_suffix_hybrid_b200.proposer import HybridProposer


def make(k=4, max_len=4096):
    return HybridProposer(SimpleNamespace(speculative_config=SimpleNamespace(num_speculative_tokens=k),
                                          model_config=SimpleNamespace(max_model_len=max_len)))


@pytest.fixture(autouse=True)
def clean_env(monkeypatch):
    for k in list(os.environ):
        if k.startswith("SUFFIX_HYBRID"):
            monkeypatch.delenv(k)
    monkeypatch.setenv("SUFFIX_HYBRID_LOG_INTERVAL", "1000000")
    monkeypatch.setenv("SUFFIX_HYBRID_NGRAM_MIN", "3")
    monkeypatch.setenv("SUFFIX_HYBRID_NGRAM_MAX", "6")


def step(p, rows, width=512, dtype=np.int64, sampled=None):
    """One propose call over Python rows; every row sampled one token unless told otherwise."""
    buf = np.full((max(len(rows), 1), width), -1, dtype=dtype)
    for i, r in enumerate(rows):
        buf[i, :len(r)] = r
    if sampled is None:
        sampled = [[r[-1]] for r in rows]
    return p.propose(sampled, np.array([len(r) for r in rows], dtype=dtype), buf)


def unique_tokens(rng, n, lo=1000, hi=50000):
    return [int(t) for t in rng.choice(np.arange(lo, hi), size=n, replace=False)]


@pytest.mark.parametrize("offset", [3, 5, 8, 13, 20])
def test_repeat_inside_a_row_is_continued(offset):
    # A run of distinct tokens followed by a partial replay of itself: the
    # only earlier occurrence of the row's tail is inside the first run, so
    # the n-gram draft must be the tokens that followed it there.
    rng = np.random.default_rng(offset)
    base = unique_tokens(rng, 40)
    row = base + base[:offset]
    p = make(k=4)
    assert step(p, [row]) == [base[offset:offset + 4]]
    assert p.get_stats()["ngram_proposals"] == 1


def test_draft_length_respects_k_and_context_limit():
    rng = np.random.default_rng(1)
    base = unique_tokens(rng, 30)
    for k in (1, 2, 6):
        assert [len(d) for d in step(make(k=k), [base + base[:10]])] == [k]
    row = base + base[:10]
    for room in (0, 1, 3):
        p = make(k=6, max_len=len(row) + room)
        assert len(step(p, [row])[0]) == room


def test_rows_without_a_sampled_token_get_no_draft():
    rng = np.random.default_rng(2)
    base = unique_tokens(rng, 25)
    rows = [base + base[:6], base[::-1] + base[::-1][:6]]
    out = step(make(), rows, sampled=[[], [rows[1][-1]]])
    assert out[0] == [] and len(out[1]) == 4


def test_continuing_rows_keep_state_in_any_order():
    rng = np.random.default_rng(3)
    a, b, c = unique_tokens(rng, 50), unique_tokens(rng, 50, 60000, 90000), unique_tokens(rng, 50, 100000, 140000)
    p = make()
    step(p, [a[:20], b[:20], c[:20]])
    for n in (23, 31, 40):  # grow every row by a different amount and shuffle the batch each time
        order = rng.permutation(3)
        step(p, [[a, b, c][i][:n + int(i)] for i in order])
        assert p.suffix_cache.stats()["num_sequences"] == 0  # nothing left the batch
    assert p.get_stats()["active_context_tokens"] == (40 + 0) + (40 + 1) + (40 + 2)


def test_finished_rows_feed_the_corpus():
    rng = np.random.default_rng(4)
    done = unique_tokens(rng, 64)
    p = make(k=5)
    step(p, [done, unique_tokens(rng, 10, 70000, 80000)])
    step(p, [])  # both rows leave the batch
    st = p.suffix_cache.stats()
    assert st["num_sequences"] == 2 and st["cached_tokens"] == 64 + 10
    # A new request that replays a stretch of the finished one is continued from the corpus.
    newcomer = unique_tokens(rng, 7, 90000, 95000) + done[17:29]
    assert step(p, [newcomer]) == [done[29:34]]
    assert p.get_stats()["suffix_proposals"] == 1


def test_a_rewritten_row_is_a_new_request():
    rng = np.random.default_rng(5)
    first = unique_tokens(rng, 30)
    p = make()
    step(p, [first])
    changed = list(first)
    changed[0] += 1  # same length, different head: not a continuation
    step(p, [changed + [7]])
    st = p.suffix_cache.stats()
    assert st["num_sequences"] == 1 and st["cached_tokens"] == 30


def test_buffer_layouts_agree():
    rng = np.random.default_rng(6)
    base = unique_tokens(rng, 30, 1000, 30000)
    row = base + base[:9]
    want = step(make(), [row])
    assert step(make(), [row], dtype=np.int32) == want
    wide = np.zeros((1, 2 * len(row)), dtype=np.int32)
    wide[0, ::2] = row  # a strided view of a wider buffer
    assert make().propose([[row[-1]]], np.array([len(row)], np.int32), wide[:, ::2]) == want


def test_bad_shapes_raise_and_leave_state_alone():
    p = make()
    step(p, [[1, 2, 3, 4, 5]])
    before = p.get_stats()
    for counts in ([-2], [600], [3, 3]):
        with pytest.raises(ValueError):
            p.propose([[1]] * len(counts), np.array(counts, np.int64), np.zeros((1, 512), np.int64))
    with pytest.raises(ValueError):
        p.propose([[1]], [5], np.zeros((1, 8), np.int64))  # counts must be an array
    after = p.get_stats()
    assert after["calls"] == before["calls"] and after["active_requests"] == 1


def test_stats_never_claim_acceptance():
    p = make()
    step(p, [[9, 8, 7, 9, 8]])
    st = p.get_stats()
    assert st["accepted"] is None and st["acceptance_rate"] is None
    assert 0 < st["native_time_ns"] <= st["total_proposer_time_ns"]


def test_stats_file_cadence(tmp_path, monkeypatch):
    path = tmp_path / "proposer.jsonl"
    monkeypatch.setenv("SUFFIX_HYBRID_STATS_FILE", str(path))
    monkeypatch.setenv("SUFFIX_HYBRID_STATS_INTERVAL", "3")
    p = make()
    for n in range(1, 8):
        step(p, [list(range(100, 100 + n + 4))])
    recs = [json.loads(line) for line in path.read_text().splitlines()]
    assert [r["calls"] for r in recs] == [3, 6]
    assert all("ts" in r and "cache" in r for r in recs)


def test_log_line_cadence(caplog, monkeypatch):
    monkeypatch.setenv("SUFFIX_HYBRID_LOG_INTERVAL", "2")
    p = make()
    with caplog.at_level("INFO", logger="suffix_hybrid"):
        for n in range(5):
            step(p, [list(range(10, 16 + n))])
    lines = [r.getMessage() for r in caplog.records if r.getMessage().startswith("suffix_hybrid {")]
    assert len(lines) == 2


def test_compat_alias_package():
    from suffix_hybrid._native import VERSION, Engine  # noqa: F401
    from suffix_hybrid.hybrid_proposer import HybridProposer as Alias
    from suffix_hybrid.suffix_cache import SuffixCache  # noqa: F401
    assert Alias is HybridProposer
