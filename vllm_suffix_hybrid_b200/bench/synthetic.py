"""Synthetic token streams with cross- and in-request span reuse.

Generator of the benchmark workloads: a row is a concatenation of segments;
with probability ``p_copy`` a segment copies a random span (length U[16,256])
from earlier in the same row or from a shared corpus of ``corpus_n``
sequences (each ``corpus_len`` Zipf(1.1) tokens), otherwise it emits 32-128
i.i.d. Zipf(1.1) tokens.  Deterministic for a seed (identical on every rank).
"""
from __future__ import annotations

import numpy as np


def zipf_tokens(rng: np.random.Generator, n: int, vocab: int, a: float = 1.1) -> np.ndarray:
    return ((rng.zipf(a, n) - 1) % vocab).astype(np.int64)


def make_streams(rows: int, length: int, vocab: int, seed: int = 0, p_copy: float = 0.4, corpus_n: int = 64,
                 corpus_len: int = 4096) -> np.ndarray:
    rng = np.random.default_rng(seed)
    corpus = [zipf_tokens(rng, corpus_len, vocab) for _ in range(corpus_n)]
    out = np.zeros((rows, length), dtype=np.int64)
    for r in range(rows):
        buf = np.zeros(length + 256, dtype=np.int64)
        n = 0
        while n < length:
            if rng.random() < p_copy:
                span = int(rng.integers(16, 257))
                if n > span and rng.random() < 0.5:  # earlier in the same row
                    s = int(rng.integers(0, n - span))
                    seg = buf[s:s + span].copy()
                else:  # shared corpus
                    c = corpus[int(rng.integers(0, corpus_n))]
                    s = int(rng.integers(0, corpus_len - span))
                    seg = c[s:s + span]
            else:
                seg = zipf_tokens(rng, int(rng.integers(32, 129)), vocab)
            m = min(len(seg), len(buf) - n)
            buf[n:n + m] = seg[:m]
            n += m
        out[r] = buf[:length]
    return out
