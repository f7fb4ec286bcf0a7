"""Host reference of the fp8 lightning indexer: page layout, quantisation, causal rows, tie rule."""
import torch

from vllm_suffix_hybrid_b200 import ops
from vllm_suffix_hybrid_b200.ops import reference as ref


def test_page_layout_round_trip():
    """Keys land as e4m3 codes at row (slot % 64) of page (slot // 64), the f32 scale after the 8192 key bytes,
    and read back within e4m3 rounding (relative 2**-4)."""
    gen = torch.Generator().manual_seed(0)
    k = torch.randn(10, 128, generator=gen) * 5
    slots = torch.tensor([0, 63, 64, 130, 191, 7, 8, 9, -1, 100])
    cache = torch.zeros(4, ops.DSA_PAGE_BYTES, dtype=torch.uint8)
    ref.dsa_cache_write(cache, k, slots)
    keys, scales = ref.dsa_keys(cache)
    for t, s in enumerate(slots.tolist()):
        if s < 0:
            continue
        back = keys[s // 64, s % 64] * scales[s // 64, s % 64]
        assert torch.allclose(back, k[t], rtol=2 ** -4, atol=scales[s // 64, s % 64].item() * 2 ** -9)
        assert abs(scales[s // 64, s % 64].item() - k[t].abs().max().item() / 448) < 1e-6 * k[t].abs().max().item()
    assert cache[3].eq(0).all()  # nothing written to an untouched page
    assert ops.DSA_PAGE_BYTES == 64 * 132


def test_zero_key_has_unit_scale():
    cache = torch.zeros(1, ops.DSA_PAGE_BYTES, dtype=torch.uint8)
    ref.dsa_cache_write(cache, torch.zeros(1, 128), torch.tensor([5]))
    keys, scales = ref.dsa_keys(cache)
    assert scales[0, 5].item() == 1.0 and keys[0, 5].eq(0).all()


def _single_request(n, IH=4, seed=1):
    gen = torch.Generator().manual_seed(seed)
    pages = (n + 63) // 64
    cache = torch.zeros(pages, ops.DSA_PAGE_BYTES, dtype=torch.uint8)
    ref.dsa_cache_write(cache, torch.randn(n, 128, generator=gen), torch.arange(n))
    bt = torch.arange(pages, dtype=torch.int32)[None]
    qi = torch.randn(2, IH, 128, generator=gen)
    w = torch.rand(2, IH, generator=gen)
    return cache, bt, qi, w, torch.tensor([n]), torch.tensor([0, 2])


def test_rows_are_causal_and_selection_is_ascending():
    cache, bt, qi, w, sl, qs = _single_request(200)
    rows = ref.dsa_logits(qi, w, cache, bt, sl, qs)
    assert [r.shape[0] for r in rows] == [199, 200]  # the last two positions are the queries
    top = ref.dsa_topk(qi, w, cache, bt, sl, qs, 16)
    for t, r in enumerate(rows):
        sel = top[t].tolist()
        assert sel == sorted(sel) and len(set(sel)) == 16
        assert set(sel) == set(torch.topk(r, 16).indices.tolist())


def test_short_context_selects_every_key():
    cache, bt, qi, w, sl, qs = _single_request(10)
    top = ref.dsa_topk(qi, w, cache, bt, sl, qs, 16)
    assert top[0].tolist() == list(range(9)) + [-1] * 7
    assert top[1].tolist() == list(range(10)) + [-1] * 6


def test_equal_logits_prefer_later_positions():
    """Identical keys give identical logits: the selection keeps the latest of them."""
    n = 100
    cache = torch.zeros(2, ops.DSA_PAGE_BYTES, dtype=torch.uint8)
    k = torch.ones(n, 128)
    k[10] = 2.0  # one key above the rest (same codes, larger scale)
    ref.dsa_cache_write(cache, k, torch.arange(n))
    bt = torch.arange(2, dtype=torch.int32)[None]
    qi = torch.ones(1, 4, 128)
    w = torch.ones(1, 4)
    top = ref.dsa_topk(qi, w, cache, bt, torch.tensor([n]), torch.tensor([0, 1]), 5)
    assert top[0].tolist() == [10, 96, 97, 98, 99]
