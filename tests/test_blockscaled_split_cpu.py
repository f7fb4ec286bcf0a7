"""Split-K choice of the dense block-scaled (W4A4 / MXFP8) GEMMs: K splits while the tiles cover at most
half the SMs and each split keeps at least 1536 of K; batch-invariant mode counts weight tiles only."""
import pytest

from vllm_suffix_hybrid_b200 import ops


@pytest.fixture
def split(monkeypatch):
    monkeypatch.setattr(ops, "_num_sms", lambda dev: 148)
    monkeypatch.setattr(ops, "workspace", lambda dev, n: ("ws", n), raising=False)
    import vllm_suffix_hybrid_b200.ops.gemm as g

    monkeypatch.setattr(g, "workspace", lambda dev, n: ("ws", n))
    monkeypatch.setattr(ops, "split_tickets", lambda dev, n: ("tickets", n))
    return lambda N, M, K, bn=64: ops._blockscaled_split("cpu", N, M, K, bn)


@pytest.mark.parametrize("N,M,K,want", [
    (4096, 64, 7168, 4),     # expert gate_up: measured 20.4 -> 16.1 us
    (7168, 64, 2048, 1),     # expert down: split 2 measured slower
    (1536, 24, 7168, 4),     # DeepSeek q_a at a rank's 24 tokens
    (7168, 24, 16384, 2),    # o_proj
    (24576, 192, 1536, 1),   # enough tiles already
    (4096, 64, 256, 1),      # one k-block
])
def test_split_rule(split, N, M, K, want):
    s, ws, cnt = split(N, M, K)
    assert s == want
    if s > 1:
        tiles = -(-N // 128) * -(-M // 64)
        assert ws == ("ws", s * tiles * 128 * 64) and cnt == ("tickets", tiles)
    else:
        assert ws is None and cnt is None


def test_split_off_switch_and_batch_invariance(split, monkeypatch):
    monkeypatch.setenv("SH_FP4_SPLITK", "0")
    assert split(4096, 64, 7168)[0] == 1
    monkeypatch.delenv("SH_FP4_SPLITK")
    monkeypatch.setenv("SH_BATCH_INVARIANT", "1")
    # the split depends on the weight tiles only: the same for 8 and 512 tokens
    assert split(4096, 8, 7168)[0] == split(4096, 512, 7168, 128)[0] == 4
