"""Suffix corpus semantics: lookup, back-extension, voting, caps, eviction.

Conformance data.  The tests from the empty corpus through the lookback
window, plus the tuple/NumPy input and concurrency tests, restate cases of
the reference's corpus suite (reference: tests/test_suffix_cache.py:31-180)
with its literal token vectors, so both implementations agree on the same
inputs; they form a conformance table.  The token-budget, churn,
positions-cap and re-index tests and the randomized comparison against a
Python oracle of the documented semantics are this package's own.
"""
import os
import threading

import numpy as np
import pytest

from vllm_suffix_hybrid_b200._native import SuffixCache


@pytest.fixture(autouse=True)
def clean_env():
    saved = {k: v for k, v in os.environ.items() if k.startswith("SUFFIX_HYBRID")}
    for k in list(saved):
        if k != "SUFFIX_HYBRID_INDEX_N":
            del os.environ[k]
    os.environ["SUFFIX_HYBRID_INDEX_N"] = "2"
    yield
    for k in [k for k in os.environ if k.startswith("SUFFIX_HYBRID")]:
        del os.environ[k]
    os.environ.update(saved)


def test_empty_corpus_has_no_draft():
    assert SuffixCache().speculate([1, 2, 3, 4, 5, 6, 7, 8], 4) == ([], 0.0, 0)


def test_continuation_of_indexed_sequence():
    c = SuffixCache()
    c.add_sequence(list(range(10, 30)))
    draft, score, matched = c.speculate([99, 12, 13, 14, 15, 16, 17, 18, 19], 3)
    assert draft == [20, 21, 22]
    assert 0.0 < score <= 1.0
    assert matched >= 8


def test_draft_capped_by_match_length_and_offset():
    c = SuffixCache()
    seq = list(range(30))
    c.add_sequence(seq)
    d, _, m = c.speculate(seq[:12], 100)
    assert len(d) <= m
    os.environ["SUFFIX_HYBRID_MAX_SPEC_OFFSET"] = "4"
    c2 = SuffixCache()
    c2.add_sequence(seq)
    d2, _, m2 = c2.speculate(seq[:12], 100)
    assert 0 < len(d2) <= m2 + 4


def test_longest_backward_match_wins():
    c = SuffixCache()
    c.add_sequence([1, 1, 1, 1, 2, 3, 4, 5, 6, 7, 8, 9])
    c.add_sequence([9, 9, 9, 9, 2, 3, 4, 5, 6, 7, 8, 9])
    assert c.speculate([1, 1, 1, 1, 2, 3, 4, 5, 6, 7, 8], 4)[0] == [9]


def test_majority_vote_and_recency_tiebreak():
    c = SuffixCache()
    for tail in (100, 100, 7):
        c.add_sequence([1, 2, 3, 4, 5, 6, 7, 8, tail])
    assert c.speculate([1, 2, 3, 4, 5, 6, 7, 8], 1)[0] == [100]
    # Equal support: the most recent occurrence wins.
    c2 = SuffixCache()
    c2.add_sequence([1, 2, 3, 4, 5, 6, 7, 8, 50])
    c2.add_sequence([1, 2, 3, 4, 5, 6, 7, 8, 60])
    draft, score, _ = c2.speculate([1, 2, 3, 4, 5, 6, 7, 8], 1)
    assert draft == [60]
    assert score == pytest.approx(0.5)


def test_min_token_count_floor():
    os.environ["SUFFIX_HYBRID_MIN_TOKEN_COUNT"] = "5"
    c = SuffixCache()
    c.add_sequence([1, 2, 3, 4, 5, 6, 7, 8, 42])
    assert c.speculate([1, 2, 3, 4, 5, 6, 7, 8], 2)[0] == []


def test_fifo_eviction_by_count():
    os.environ["SUFFIX_HYBRID_MAX_CACHED_REQUESTS"] = "2"
    c = SuffixCache()
    for tail in (11, 22, 33):
        c.add_sequence([1, 2, 3, 4, 5, 6, 7, 8, tail])
    assert c.speculate([1, 2, 3, 4, 5, 6, 7, 8], 1)[0] == [33]
    assert c.stats()["num_sequences"] == 2


def test_unparsable_knob_uses_default():
    os.environ["SUFFIX_HYBRID_MAX_CACHED_REQUESTS"] = "-1"
    c = SuffixCache()
    for i in range(20):
        c.add_sequence([1, 2, 3, 4, 5, 6, 7, 8, i])
    st = c.stats()
    assert st["num_sequences"] == 20 and st["max_cached_requests"] == 512


def test_short_sequences_are_not_indexed():
    c = SuffixCache()
    c.add_sequence([1, 2])  # == n
    st = c.stats()
    assert st["cached_tokens"] == 0 and st["num_sequences"] == 0 and st["num_index_keys"] == 0
    assert c.speculate([1, 2], 4) == ([], 0.0, 0)
    c.add_sequence([1, 2, 3])  # n + 1: one window
    assert c.stats()["cached_tokens"] == 3
    d, _, m = c.speculate([1, 2], 4)
    assert d == [3] and m >= 2


def test_lookback_window_is_max_tree_depth():
    os.environ["SUFFIX_HYBRID_MAX_TREE_DEPTH"] = "16"
    c = SuffixCache()
    seq = list(range(100))
    c.add_sequence(seq)
    assert c.speculate(seq[:80], 4)[0] == seq[80:84]


def test_token_budget_keeps_tail_with_exact_capacity():
    os.environ["SUFFIX_HYBRID_MAX_CACHED_TOKENS"] = "16"
    c = SuffixCache()
    c.add_sequence(list(range(100_000)))
    st = c.stats()
    assert st["cached_tokens"] == 16 and st["allocated_token_capacity"] <= 16
    assert c.speculate(list(range(99984, 99992)), 2)[0] == [99992, 99993]


def test_bounded_index_under_churn():
    os.environ["SUFFIX_HYBRID_MAX_CACHED_REQUESTS"] = "2"
    os.environ["SUFFIX_HYBRID_MAX_CACHED_TOKENS"] = "20"
    c = SuffixCache()
    for i in range(100):
        c.add_sequence(list(range(i * 20, i * 20 + 10)))
    st = c.stats()
    assert st["num_sequences"] <= 2 and st["cached_tokens"] <= 20 and st["num_index_keys"] <= 18
    assert c.speculate(list(range(8)), 2)[0] == []
    assert c.speculate(list(range(1980, 1988)), 2)[0] == [1988, 1989]


def test_positions_per_ngram_cap_keeps_newest():
    os.environ["SUFFIX_HYBRID_MAX_POSITIONS_PER_NGRAM"] = "1"
    c = SuffixCache()
    c.add_sequence([5, 6, 70, 71])
    c.add_sequence([5, 6, 80, 81])
    assert c.stats()["index_positions"] == 5  # (5,6) keeps one position
    assert c.speculate([5, 6], 2)[0] == [80, 81]


def test_set_test_n_reindexes():
    os.environ["SUFFIX_HYBRID_INDEX_N"] = "8"
    c = SuffixCache()
    c.add_sequence(list(range(20)))
    assert c.speculate([3, 4], 2)[0] == []
    c.set_test_n(2)
    assert c.stats()["index_n"] == 2
    assert c.speculate([3, 4], 2)[0] == [5, 6]


def test_accepts_tuples_and_numpy():
    c = SuffixCache()
    c.add_sequence((1, 2, 3, 4, 5, 6, 7, 8, 9))
    assert c.speculate(np.arange(1, 9, dtype=np.int64), 1)[0] == [9]
    c.add_sequence(np.array([40, 41, 42], dtype=np.int32))
    assert c.speculate((40, 41), 1)[0] == [42]


def test_concurrent_readers_and_writers():
    c = SuffixCache()
    errors = []

    def writer(base):
        try:
            for i in range(200):
                c.add_sequence([base + j for j in range(8)] + [i])
        except Exception as e:  # pragma: no cover
            errors.append(e)

    def reader():
        try:
            for _ in range(200):
                c.speculate([1, 2, 3, 4, 5, 6, 7, 8], 2)
        except Exception as e:  # pragma: no cover
            errors.append(e)

    ts = [threading.Thread(target=writer, args=(b,)) for b in (1, 100)] + [threading.Thread(target=reader) for _ in range(2)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert errors == []


def _python_oracle(corpus, context, max_tokens, n, depth=64, cands=32, positions=64):
    """Straight-line Python restatement of the corpus lookup (test oracle)."""
    index = {}
    for sid, seq in enumerate(corpus):
        if len(seq) <= n:
            continue
        for pos in range(len(seq) - n + 1):
            b = index.setdefault(tuple(seq[pos:pos + n]), [])
            b.append((sid, pos))
            if len(b) > positions:
                b.pop(0)
    window = context[-depth:]
    if max_tokens == 0 or len(window) < n:
        return [], 0.0, 0
    bucket = index.get(tuple(window[-n:]))
    if not bucket:
        return [], 0.0, 0
    best, ends = 0, []
    for sid, pos in list(reversed(bucket))[:cands]:
        s = corpus[sid]
        m = n
        while m < len(window) and m < pos + n and s[pos + n - m - 1] == window[-m - 1]:
            m += 1
        if m > best:
            best, ends = m, []
        if m == best:
            ends.append((sid, pos + n))
    cap = min(max_tokens, int(max(0.0, 1.0 * best)))
    out, score = [], 1.0
    for step in range(cap):
        votes = {}
        for sid, pos in ends:
            s = corpus[sid]
            if pos + step < len(s):
                t = s[pos + step]
                sup, bid, bpos = votes.get(t, (0, sid, pos))
                if (sid, pos) > (bid, bpos):
                    bid, bpos = sid, pos
                votes[t] = (sup + 1, bid, bpos)
        if not votes:
            break
        tok, (sup, _, _) = max(votes.items(), key=lambda kv: (kv[1], kv[0]))
        score *= sup / len(ends)
        out.append(tok)
        ends = [(sid, pos) for sid, pos in ends if pos + step < len(corpus[sid]) and corpus[sid][pos + step] == tok]
    return out, (score if out else 0.0), best


def test_randomized_against_python_oracle():
    rng = np.random.default_rng(0)
    for trial in range(60):
        vocab = int(rng.integers(3, 12))
        corpus = [list(map(int, rng.integers(0, vocab, int(rng.integers(3, 60))))) for _ in range(int(rng.integers(1, 8)))]
        c = SuffixCache()
        for s in corpus:
            c.add_sequence(s)
        for _ in range(10):
            ctx = list(map(int, rng.integers(0, vocab, int(rng.integers(1, 40)))))
            k = int(rng.integers(0, 8))
            got = c.speculate(ctx, k)
            want = _python_oracle(corpus, ctx, k, 2)
            assert got[0] == want[0] and got[2] == want[2], (trial, ctx)
            assert got[1] == pytest.approx(want[1])
