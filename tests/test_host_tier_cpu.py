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
