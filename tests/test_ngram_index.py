"""The incremental n-gram index returns exactly what the backward scan does."""
import os

import numpy as np
import pytest

from vllm_suffix_hybrid_b200._native import Engine


def scan(ctx, lo, hi, cap, window):
    """Python restatement of the in-request lookup (oracle)."""
    if cap == 0 or not ctx:
        return []
    hi = min(hi, len(ctx) - 1)
    if hi < lo:
        return []
    L = len(ctx)
    qmax = L if window == 0 else min(window, L)
    latest = {}
    for q in range(1, qmax):
        l = 0
        while l < hi and q + l < L and ctx[L - 1 - q - l] == ctx[L - 1 - l]:
            l += 1
        for n in range(lo, min(l, hi) + 1):
            latest.setdefault(n, L - n - q)
        if hi in latest:
            break
    for n in range(hi, lo - 1, -1):
        if n in latest:
            pos = latest[n]
            return ctx[pos + n:min(pos + n + cap, L)]
    return []


@pytest.mark.parametrize("window", [0, 7, 40])
def test_growing_rows_match_scan(window):
    saved = dict(os.environ)
    try:
        os.environ.update({"SUFFIX_HYBRID_NGRAM_MIN": "2", "SUFFIX_HYBRID_NGRAM_MAX": "5",
                           "SUFFIX_HYBRID_USE_NGRAM": "1", "SUFFIX_HYBRID_NGRAM_WINDOW": str(window),
                           "SUFFIX_HYBRID_MAX_CACHED_REQUESTS": "0"})  # corpus off: n-gram only
        rng = np.random.default_rng(window)
        e = Engine(4, 4096)
        rows = [list(map(int, rng.integers(0, 4, 5))) for _ in range(3)]
        for step in range(80):
            for r in rows:
                r.extend(map(int, rng.integers(0, 4, int(rng.integers(1, 4)))))
            buf = np.zeros((3, 4096), dtype=np.int64)
            for i, r in enumerate(rows):
                buf[i, :len(r)] = r
            got = e.propose([[1]] * 3, np.array([len(r) for r in rows], dtype=np.int64), buf)
            want = [scan(r, 2, 5, 4, window) for r in rows]
            assert got == want, step
    finally:
        os.environ.clear()
        os.environ.update(saved)
