"""Hybrid mixer (legacy split): learned native budget + conditioned suffix tail.

Conformance data.  The first nine tests (fresh row .. cache tokens on
departure) restate cases of the reference's own mixer suite
(reference: tests/test_mixer.py:6-110) with the same literal token
vectors, so this implementation and the reference give the same drafts and
counters on the same inputs; they are kept as a conformance table, not as
independent design.  The tests after them (incremental NumPy rows, id
reuse, shrinking rows, boundary windows, int32 rows, default split) and the
randomized tests in test_mixer_diverge.py are this package's own.
"""
import os

import numpy as np
import pytest

from vllm_suffix_hybrid_b200._native import HybridMixer


@pytest.fixture(autouse=True)
def env():
    saved = {k: v for k, v in os.environ.items() if k.startswith("SUFFIX_HYBRID")}
    for k in list(saved):
        del os.environ[k]
    os.environ["SUFFIX_HYBRID_INDEX_N"] = "2"
    yield
    for k in [k for k in os.environ if k.startswith("SUFFIX_HYBRID")]:
        del os.environ[k]
    os.environ.update(saved)


def buf(rows, width, seqs, dtype=np.int64):
    d = np.zeros((rows, width), dtype=dtype)
    for i, s in enumerate(seqs):
        d[i, :len(s)] = s
    return d


def test_fresh_row_is_native_then_tail_replaces():
    m = HybridMixer(5, 128)
    m.suffix_cache.add_sequence(list(range(1, 30)))
    assert m.mix(["a"], [list(range(1, 9))], [[9, 10, 11, 12, 99]], None) == [[9, 10, 11, 12, 99]]
    assert m.last_native_counts() == [5]
    assert m.mix(["a"], [list(range(1, 9))], [[9, 10, 11, 12, 99]], [5]) == [[9, 10, 11, 12, 13]]
    assert m.last_native_counts() == [4]


def test_without_corpus_native_is_published_whole():
    m = HybridMixer(5, 128)
    assert m.mix(["a"], [[1, 2]], [[3, 4, 5, 6, 7]], None) == [[3, 4, 5, 6, 7]]
    assert m.last_native_counts() == [5]


def test_feedback_counts_only_reached_positions():
    m = HybridMixer(5, 128)
    m.suffix_cache.add_sequence(list(range(1, 30)))
    m.mix(["a"], [list(range(1, 9))], [[9, 10, 11, 12, 99]], None)
    m.mix(["a"], [list(range(1, 11))], [[11, 12, 13, 14, 99]], [1])
    st = m.get_stats()
    assert (st["native_tested"], st["native_accepted"], st["suffix_tested"]) == (2, 1, 0)


def test_budget_tracks_row_acceptance():
    m = HybridMixer(5, 128)
    m.suffix_cache.add_sequence(list(range(1, 100)))
    native = [[9, 10, 11, 99, 98]]
    acc = None
    for _ in range(10):
        m.mix(["a"], [list(range(1, 9))], native, acc)
        acc = [2]
    got = m.mix(["a"], [list(range(1, 9))], native, [2])
    assert m.last_native_counts()[0] <= 4
    assert len(got[0]) == 5 and got[0][:2] == [9, 10] and got[0][3:] != [99, 98]
    b_acc = None
    for _ in range(12):
        got_b = m.mix(["b"], [list(range(1, 9))], [[9, 10, 11, 12, 13]], b_acc)
        b_acc = [5]
    assert got_b == [[9, 10, 11, 12, 13]] and m.last_native_counts()[0] == 5


def test_numpy_rows_both_dtypes():
    m = HybridMixer(5, 128)
    m.suffix_cache.add_sequence(list(range(1, 30)))
    for dtype in (np.int32, np.int64):
        data = np.arange(1, 257, dtype=dtype).reshape(1, -1)
        got = m.mix_numpy(["a"], np.array([8], dtype=dtype), data, [[9, 10, 11, 12, 99]], None)
        assert got[0][:4] == [9, 10, 11, 12]
    with pytest.raises(ValueError):
        m.mix_numpy(["a"], np.array([-1], dtype=np.int32), data, [[9]], None)


def test_rejected_batches_leave_state_untouched():
    m = HybridMixer(4, 128)
    with pytest.raises(ValueError):
        m.mix(["a"], [], [[1, 2]], None)
    with pytest.raises(ValueError):
        m.mix(["a", "a"], [[1], [1]], [[2], [2]], None)
    with pytest.raises(ValueError):
        m.mix(["a"], [[1]], [[1, 2, 3, 4, 5]], None)  # wider than k
    with pytest.raises(ValueError):
        m.mix(["a"], [[1]], [[-3]], None)  # negative token
    assert m.get_stats()["calls"] == 0
    m.mix(["a"], [[1, 2]], [[3, 4]], None)
    with pytest.raises(ValueError, match="accepted length"):
        m.mix(["a"], [[1, 2, 3]], [[3, 4]], [3])  # more than published
    assert m.get_stats()["calls"] == 1


def test_context_limit_caps_draft():
    m = HybridMixer(5, 10)
    assert m.mix(["a"], [list(range(9))], [[9, 10, 11]], None) == [[9]]


def test_constructor_bounds():
    with pytest.raises(ValueError):
        HybridMixer(0, 10)
    with pytest.raises(ValueError):
        HybridMixer(65, 10)


def test_cache_tokens_grows_on_departure():
    m = HybridMixer(4, 128)
    assert m.cache_tokens() == 0
    acc = None
    for step in range(4):
        ctx = list(range(1, 10 + step))
        m.mix(["a", "b"], [ctx, [x + 100 for x in ctx]], [[10, 11, 12, 13], [14, 15, 16, 17]], acc)
        acc = [2, 2]
    assert m.cache_tokens() == 0
    m.mix(["a"], [list(range(1, 14))], [[10, 11, 12, 13]], [2])
    assert m.cache_tokens() > 0


def test_numpy_incremental_equals_list_api():
    corpus = list(range(1, 40))
    native = [[40, 41, 42, 43, 99]]
    a, b = HybridMixer(5, 128), HybridMixer(5, 128)
    a.suffix_cache.add_sequence(corpus)
    b.suffix_cache.add_sequence(corpus)
    for step, n in enumerate([8, 9, 10, 11, 12]):
        acc = None if step == 0 else [5]
        want = a.mix(["a"], [corpus[:n]], native, acc)
        got = b.mix_numpy(["a"], np.array([n], dtype=np.int64), buf(1, 64, [corpus[:n]]), native, acc)
        assert got == want and b.last_native_counts() == a.last_native_counts()


def test_reused_id_resets_to_native():
    m = HybridMixer(5, 128)
    m.suffix_cache.add_sequence(list(range(1, 30)))
    m.mix_numpy(["a"], np.array([8]), buf(1, 64, [list(range(1, 9))]), [[9, 10, 11, 12, 99]], None)
    got = m.mix_numpy(["a"], np.array([4]), buf(1, 64, [[100, 101, 102, 103]]), [[104, 105, 106, 107, 108]], None)
    assert got == [[104, 105, 106, 107, 108]]
    assert m.get_stats()["cache"]["num_sequences"] > 0


def test_shrinking_row_resets():
    m = HybridMixer(4, 128)
    m.mix_numpy(["a"], np.array([16]), buf(1, 64, [list(range(1, 20))]), [[1, 2, 3, 4]], None)
    assert m.mix_numpy(["a"], np.array([3]), buf(1, 64, [[7, 8, 9]]), [[5, 6]], None) == [[5, 6]]


def test_boundary_windows_detect_long_continuations():
    m = HybridMixer(3, 4096)
    base = list(range(1, 200))
    m.mix_numpy(["a"], np.array([len(base)]), buf(1, 512, [base]), [[900, 901, 902]], None)
    grown = base + [900, 901]
    got = m.mix_numpy(["a"], np.array([len(grown)]), buf(1, 512, [grown]), [[903, 904, 905]], [3])
    assert got == [[903, 904, 905]] and m.get_stats()["active_tracked"] == 1


def test_int32_rows_incremental():
    corpus = list(range(1, 30))
    m = HybridMixer(4, 128)
    m.suffix_cache.add_sequence(corpus)
    for n in (8, 10, 12):
        d = np.zeros((1, 64), dtype=np.int32)
        d[0, :n] = corpus[:n]
        assert m.mix_numpy(["a"], np.array([n], dtype=np.int32), d, [[30, 31, 32, 33]], None) == [[30, 31, 32, 33]]


def test_legacy_is_default_split():
    assert HybridMixer(5, 128).get_stats()["split_mode"] == "legacy"
