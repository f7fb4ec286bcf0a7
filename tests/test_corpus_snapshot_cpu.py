"""Suffix corpus snapshot / restore: the corpus survives a restart.

A snapshot holds the corpus's sequences oldest first (native `save_corpus`); restoring adds them through
the normal ingest path, so a restored corpus drafts exactly what the saved one drafted.  A damaged file is
rejected whole before anything is added.
"""
import os

import numpy as np
import pytest

from vllm_suffix_hybrid_b200 import _native


def _filled(seed=0, n=40):
    rng = np.random.default_rng(seed)
    c = _native.SuffixCache()
    seqs = []
    for _ in range(n):
        base = rng.integers(0, 50, 30).tolist()
        s = base + base[:10] + rng.integers(0, 50, int(rng.integers(5, 40))).tolist()
        c.add_sequence(s)
        seqs.append(s)
    return c, seqs


def _drafts(c, seqs):
    return [c.speculate(s[: 12 + i % 7], 6) for i, s in enumerate(seqs)]


def test_restore_drafts_like_the_saved_corpus(tmp_path):
    c, seqs = _filled()
    path = str(tmp_path / "corpus.bin")
    assert c.save(path) == c.stats()["num_sequences"] == 40
    assert not os.path.exists(path + ".tmp")
    r = _native.SuffixCache()
    assert r.load(path) == 40
    for key in ("num_sequences", "cached_tokens", "num_index_keys", "index_positions"):
        assert r.stats()[key] == c.stats()[key], key
    assert _drafts(r, seqs) == _drafts(c, seqs)


def test_save_replaces_the_previous_snapshot(tmp_path):
    path = str(tmp_path / "corpus.bin")
    a, _ = _filled(1, 10)
    a.save(path)
    b, seqs = _filled(2, 25)
    b.save(path)
    r = _native.SuffixCache()
    assert r.load(path) == 25
    assert _drafts(r, seqs) == _drafts(b, seqs)


@pytest.mark.parametrize("damage", ["flip", "truncate", "magic", "empty"])
def test_damaged_snapshot_is_rejected_before_any_change(tmp_path, damage):
    c, _ = _filled(3, 12)
    path = str(tmp_path / "corpus.bin")
    c.save(path)
    data = bytearray(open(path, "rb").read())
    if damage == "flip":
        data[len(data) // 2] ^= 0x40
    elif damage == "truncate":
        data = data[: len(data) - 20]
    elif damage == "magic":
        data[0:8] = b"NOTACORP"
    else:
        data = bytearray()
    open(path, "wb").write(bytes(data))
    r, _ = _filled(4, 5)
    before = r.stats()
    with pytest.raises(RuntimeError, match="suffix corpus restore"):
        r.load(path)
    assert r.stats() == before
    with pytest.raises(RuntimeError, match="cannot open"):
        r.load(str(tmp_path / "missing.bin"))


def test_restore_respects_the_corpus_bounds(tmp_path, monkeypatch):
    c, _ = _filled(5, 40)
    path = str(tmp_path / "corpus.bin")
    c.save(path)
    monkeypatch.setenv("SUFFIX_HYBRID_MAX_CACHED_REQUESTS", "16")
    small = _native.SuffixCache()
    assert small.load(path) == 40  # every sequence went through ingest; the oldest were evicted
    assert small.stats()["num_sequences"] == 16


def test_engine_restores_its_corpus_at_start(tmp_path, monkeypatch):
    from vllm_suffix_hybrid_b200.engine.config import (CacheConfig, EngineConfig, SpecConfig, llama3_8b_config,
                                                       shrink)
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine

    m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=256)

    def cfg():
        return EngineConfig(model=m, spec=SpecConfig(method="hybrid", k=3), cache=CacheConfig(max_model_len=256),
                            max_num_seqs=4, device="cpu", cuda_graphs=False)

    eng = LLMEngine(cfg())
    rng = np.random.default_rng(9)
    eng.warm_start([rng.integers(0, 256, 60).tolist() for _ in range(6)])
    path = str(tmp_path / "corpus.bin")
    assert eng.save_corpus(path) == 6
    monkeypatch.setenv("SUFFIX_HYBRID_CORPUS_FILE", path)
    eng2 = LLMEngine(cfg())
    assert eng2.proposer.suffix_cache.stats()["num_sequences"] == 6
    assert eng2.proposer.suffix_cache.stats()["cached_tokens"] == eng.proposer.suffix_cache.stats()["cached_tokens"]
    eng2.warm_start([rng.integers(0, 256, 60).tolist()])
    assert eng2.save_corpus() == 7  # default path: SUFFIX_HYBRID_CORPUS_FILE
