"""Host KV tier (HiSparse): knobs, sizing and the configurations that refuse it (CPU)."""
import pytest

from vllm_suffix_hybrid_b200.engine.config import (CacheConfig, EngineConfig, SpecConfig, apply_env,
                                                   deepseek_v32_config, llama3_8b_config, shrink)
from vllm_suffix_hybrid_b200.engine.host_tier import MAX_HOT_ROWS, hot_rows_for


def test_env_knobs(monkeypatch):
    monkeypatch.setenv("SUFFIX_HYBRID_HOST_KV", "1")
    monkeypatch.setenv("SUFFIX_HYBRID_HOST_KV_HOT_ROWS", "4096")
    cfg = apply_env(EngineConfig())
    assert cfg.cache.host_kv and cfg.cache.host_kv_hot_rows == 4096
    monkeypatch.setenv("SUFFIX_HYBRID_HOST_KV", "0")
    assert not apply_env(EngineConfig()).cache.host_kv


def test_default_hot_rows_cover_one_verify_step():
    # k = 5 verify: 6 query tokens x top-2048 distinct keys at most, plus one top-k of slack, in 64-row blocks
    assert hot_rows_for(5, 2048) == 7 * 2048
    assert hot_rows_for(3, 100) % 64 == 0 and hot_rows_for(3, 100) >= 5 * 100
    assert hot_rows_for(9, 2048) == MAX_HOT_ROWS


@pytest.mark.parametrize("name", ["llama", "deepseek_cpu"])
def test_tier_is_refused_where_it_cannot_apply(name):
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine

    if name == "llama":
        m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=256)
    else:
        m = shrink(deepseek_v32_config(), layers=2, hidden=128, vocab=256)
    cfg = EngineConfig(model=m, spec=SpecConfig(method="none"), cache=CacheConfig(max_model_len=256, host_kv=True),
                       max_num_seqs=2, device="cpu")
    with pytest.raises(ValueError, match="host KV tier"):
        LLMEngine(cfg)


def _state(P=2048, H=128):
    import numpy as np

    return np.full(P, -1, dtype=np.int64), np.full(H, -1, dtype=np.int64), np.zeros(H, dtype=np.int64)


def test_reference_resolver_lru_and_rewrite():
    """The policy the kernel implements (same scenario as the GPU test): C evicts A, the least recently used,
    not B; B is then all hits; a rewritten resident position is fetched again."""
    import numpy as np

    from vllm_suffix_hybrid_b200.engine.host_tier import resolve_reference

    p2s, s2p, stp = _state()
    A, B, C = np.arange(0, 64), np.arange(100, 164), np.arange(200, 264)
    q = np.array([999])
    for tick, keys in ((1, A), (2, B)):
        out, hits, fetched, ovf = resolve_reference(p2s, s2p, stp, tick, keys[None], q)
        assert hits == 0 and len(fetched) == 64 and not ovf
        assert (s2p[out[0]] == keys).all()  # every key's row holds it
    out, hits, fetched, ovf = resolve_reference(p2s, s2p, stp, 3, C[None], q)
    assert fetched == C.tolist() and (p2s[A] == -1).all() and (p2s[B] >= 0).all()
    out, hits, fetched, ovf = resolve_reference(p2s, s2p, stp, 4, B[None], q)
    assert hits == 64 and fetched == []
    out, hits, fetched, ovf = resolve_reference(p2s, s2p, stp, 5, B[None], np.array([120]), written=[120])
    assert fetched == [120] and hits == 20  # keys 100..120 are causal; 120 was rewritten
    assert (out[0][B > 120] == -1).all()


def test_reference_resolver_dedups_and_flags_overflow():
    import numpy as np

    from vllm_suffix_hybrid_b200.engine.host_tier import resolve_reference

    p2s, s2p, stp = _state(H=64)
    keys = np.stack([np.arange(0, 64), np.arange(32, 96)])  # 96 distinct keys over two query tokens
    out, hits, fetched, ovf = resolve_reference(p2s, s2p, stp, 1, keys, np.array([500, 501]))
    assert ovf and len(fetched) == 64 and len(set(fetched)) == 64
    p2s, s2p, stp = _state(H=64)
    keys = np.stack([np.arange(0, 64), np.arange(0, 64)[::-1]])  # shared keys fetch once
    out, hits, fetched, ovf = resolve_reference(p2s, s2p, stp, 1, keys, np.array([500, 501]))
    assert not ovf and len(fetched) == 64 and (out[0] == out[1][::-1]).all()
