"""Suffix-only proposer: mirrors, echo hits, ingestion, ragged/uniform widths, width gate."""
import numpy as np
import pytest

from vllm_suffix_hybrid_b200._native import V2SuffixProposer


def b32(r=8, c=512):
    return np.zeros((r, c), dtype=np.int32)


def i64(*v):
    return np.array(v, dtype=np.int64)


def seed_a(p, tokens, seq):
    tokens[0, :len(seq)] = seq
    for t in (10, len(seq)):
        p.propose_suffix_only(["a"], i64(0), i64(t), tokens)


def test_cold_row_misses_with_2d_pack():
    p = V2SuffixProposer(4, 512)
    t = b32()
    t[0, :10] = np.arange(10)
    packed, widths = p.propose_suffix_only(["a"], i64(0), i64(10), t)
    assert widths.tolist() == [0] and packed.shape == (1, 4) and (packed == 0).all()


def test_departed_history_drafts_for_repeating_request():
    p = V2SuffixProposer(4, 512)
    t = b32()
    seq = list(range(100, 122))
    seed_a(p, t, seq)
    t[1, :10] = seq[:10]
    packed, widths = p.propose_suffix_only(["b"], i64(1), i64(10), t)
    assert widths.tolist() == [4] and packed[0].tolist() == seq[10:14]
    st = p.get_stats()
    assert (st["hits"], st["hit_tokens"], st["ingested"]) == (1, 4, 1)
    for n in (11, 12, 13):
        t[1, :n] = seq[:n]
        packed, widths = p.propose_suffix_only(["b"], i64(1), i64(n), t)
        assert widths[0] == 4 and packed[0].tolist() == seq[n:n + 4]
    assert p.get_stats()["resets"] == 0


def test_changed_content_resets_not_stitches():
    p = V2SuffixProposer(4, 512)
    t = b32()
    seed_a(p, t, list(range(100, 122)))
    other = list(range(500, 540))
    t[0, :12] = other[:12]
    _, w = p.propose_suffix_only(["c"], i64(0), i64(12), t)
    assert w[0] == 0
    p.propose_suffix_only(["c"], i64(0), i64(12), t)
    assert p.get_stats()["resets"] == 0
    t[0, :12] = np.arange(700, 712)
    p.propose_suffix_only(["c"], i64(0), i64(12), t)
    assert p.get_stats()["resets"] == 1


def test_ingestion_gate_is_longer_than_8():
    for row_len, ingested in ((8, 0), (9, 1)):
        p = V2SuffixProposer(4, 512)
        t = b32(2)
        row = list(range(100, 100 + row_len))
        t[1, :row_len] = row
        p.propose_suffix_only(["a"], i64(1), i64(row_len), t)
        p.propose_suffix_only(["b"], i64(0), i64(1), b32(2))
        assert p.get_stats()["ingested"] == ingested
        if ingested:
            t[0, :] = 0
            t[0, :6] = row[:6]
            packed, widths = p.propose_suffix_only(["c"], i64(0), i64(6), t)
            assert widths.tolist() == [3] and packed[0].tolist() == row[6:9] + [0]


def test_int64_buffer_and_multirow():
    p = V2SuffixProposer(4, 512)
    t = np.zeros((8, 512), dtype=np.int64)
    seq = list(range(100, 140))
    t[0, :22] = seq[:22]
    p.propose_suffix_only(["a"], i64(0), i64(22), t)
    t[1, :10] = seq[:10]
    t[2, :10] = np.arange(500, 510)
    packed, widths = p.propose_suffix_only(["b", "c"], i64(1, 2), i64(10, 10), t)
    assert packed.shape == (2, 4) and widths.tolist() == [4, 0]
    assert packed[0].tolist() == seq[10:14] and (packed[1] == 0).all()


def test_bad_dimensions_raise():
    p = V2SuffixProposer(4, 512)
    with pytest.raises(ValueError):
        p.propose_suffix_only(["a", "b"], i64(0), i64(10), b32())
    with pytest.raises(ValueError):
        p.propose_suffix_only(["a"], i64(99), i64(10), b32())  # row index outside buffer


def test_min_len_floor():
    p = V2SuffixProposer(4, 512, 3)
    t = b32()
    seq = list(range(100, 110))
    t[0, :10] = seq
    p.propose_suffix_only(["a"], i64(0), i64(10), t)
    t[1, :9] = seq[:9]
    _, w = p.propose_suffix_only(["b"], i64(1), i64(9), t)
    assert w.tolist() == [0]


def test_widths_table_and_clear():
    p = V2SuffixProposer(4, 512)
    t = b32()
    seq = list(range(100, 122))
    seed_a(p, t, seq)
    assert dict(p.widths_table) == {"a": 0}
    t[1, :10] = seq[:10]
    p.propose_suffix_only(["b"], i64(1), i64(10), t)
    assert p.widths_table["b"] > 0
    p.clear_widths()
    assert dict(p.widths_table) == {"b": 0}


def test_uniform_pallet_pads_with_first_token():
    p = V2SuffixProposer(4, 512, 1, True)
    t = b32()
    seq = list(range(200, 240))
    t[0, :12] = seq[:12]
    packed, widths = p.propose_suffix_only(["a"], i64(0), i64(12), t)
    assert widths.tolist() == [4] and (packed[0] == seq[0]).all()
    t[1, :10] = seq[:10]
    packed, widths = p.propose_suffix_only(["b"], i64(1), i64(10), t)
    assert widths.tolist() == [4] and packed[0].tolist() == seq[10:12] + [seq[0]] * 2
    st = p.get_stats()
    assert st["padded"] == 2 and st["hits"] == 1 and st["hit_tokens"] == 2 and st["uniform_k"] is True


# --- acceptance-EWMA width gate --------------------------------------------
K, NCOLS = 4, 384
SEQ = list(range(101, 121)) * 8


def drive(p, accepted_seq, steps):
    t = np.zeros((4, NCOLS), dtype=np.int32)
    t[0, :len(SEQ)] = SEQ
    p.propose_suffix_only(["a"], i64(0), i64(len(SEQ)), t)
    p.propose_suffix_only([], np.array([], dtype=np.int64), np.array([], dtype=np.int64), t)
    t[1, :10] = SEQ[:10]
    total, out = 10, []
    for s in range(steps):
        packed, widths = p.propose_suffix_only(["b"], i64(1), i64(total), t)
        out.append((packed.copy(), int(widths[0])))
        total += accepted_seq[s % len(accepted_seq)] + 1
        t[1, :total] = SEQ[:total]
    return out


def test_gate_narrows_under_rejection_with_floor_one():
    p = V2SuffixProposer(K, NCOLS, 1, False, True)
    widths = [w for _, w in drive(p, [0], 8)]
    assert widths == [4, 3, 2, 2, 1, 1, 1, 1]
    assert p.get_stats()["hits"] == 8
    assert p.gate_table["b"][0] == 4.0 * 0.7 ** 7


def test_gate_decay_constants():
    p = V2SuffixProposer(K, NCOLS, 1, False, True)
    drive(p, [1], 4)
    want = 4.0
    for _ in range(3):
        want = 0.7 * want + 0.3
    assert abs(p.gate_table["b"][0] - want) < 1e-12


def test_gate_full_acceptance_stays_at_k_and_recovers():
    p = V2SuffixProposer(K, NCOLS, 1, False, True)
    assert [w for _, w in drive(p, [4], 6)] == [4] * 6
    p2 = V2SuffixProposer(K, NCOLS, 1, False, True)
    widths = [w for _, w in drive(p2, [0, 0, 0, 0, 0, 1, 2, 2, 2, 2, 2, 2], 12)]
    assert all(1 <= w <= K for w in widths)


def test_gate_off_is_identical_to_default():
    a = V2SuffixProposer(K, NCOLS)
    b = V2SuffixProposer(K, NCOLS, 1, False, False)
    for (pa, wa), (pb, wb) in zip(drive(a, [0, 2], 6), drive(b, [0, 2], 6)):
        assert (pa == pb).all() and wa == wb
    assert b.get_stats()["width_gate"] is False and dict(b.gate_table) == {}


def test_clear_widths_censors_gate_feedback():
    p = V2SuffixProposer(K, NCOLS, 1, False, True)
    t = np.zeros((4, NCOLS), dtype=np.int32)
    t[0, :len(SEQ)] = SEQ
    p.propose_suffix_only(["a"], i64(0), i64(len(SEQ)), t)
    p.propose_suffix_only([], np.array([], dtype=np.int64), np.array([], dtype=np.int64), t)
    t[1, :10] = SEQ[:10]
    p.propose_suffix_only(["b"], i64(1), i64(10), t)
    before = p.gate_table["b"][0]
    p.clear_widths()
    assert p.widths_table["b"] == 0
    t[1, :12] = SEQ[:12]
    p.propose_suffix_only(["b"], i64(1), i64(12), t)
    assert p.gate_table["b"][0] == before  # retracted publish never trains
    assert p.get_stats()["resets"] == 0
