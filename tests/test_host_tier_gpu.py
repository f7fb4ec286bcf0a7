"""Host KV tier (HiSparse): the device resolver over a latent cache in mapped host memory.

The resolver must leave, for every selected key, a hot row byte-identical to the key's host row; evict the
least recently used rows first; drop the hot copy of positions a step rewrites; flag a step whose distinct
keys outnumber the hot rows; and an engine with the tier must generate exactly what it generates with the
cache on the device.
"""
import numpy as np
import pytest
import torch

from vllm_suffix_hybrid_b200 import ops
from vllm_suffix_hybrid_b200.engine.host_tier import HostKVTier
from vllm_suffix_hybrid_b200.models.common import AttnMeta

pytestmark = pytest.mark.gpu

ROW = 352  # NVFP4 latent row bytes


def _tier(H, slots=6, blocks=40, layers=1, max_tokens=16, K=64):
    return HostKVTier(layers, blocks, 64, (ROW,), torch.uint8, slots, H, 64 * blocks, max_tokens, K, "cuda")


def _meta(seqs, qlens, state_slots, bt, written=None):
    B = len(seqs)
    qs = np.concatenate([[0], np.cumsum(qlens)])
    pos = np.concatenate([np.arange(s - q, s) for s, q in zip(seqs, qlens)])
    slot_map = np.full(len(pos), -1) if written is None else np.asarray(written)
    return AttnMeta(positions=torch.tensor(pos, device="cuda"), slot_mapping=torch.tensor(slot_map, device="cuda"),
                    block_tables=bt, seq_lens=torch.tensor(seqs, device="cuda"),
                    q_start=torch.tensor(qs, device="cuda"), tile_req=torch.zeros(1, dtype=torch.int32),
                    tile_row0=torch.zeros(1, dtype=torch.int32), num_tokens=len(pos),
                    state_slots=torch.tensor(state_slots, device="cuda"), window=max(qlens))


def _fill_cold(tier, gen):
    for c in tier.cold:
        c.copy_(torch.randint(0, 256, tuple(c.shape), dtype=torch.uint8, generator=gen).cuda())


def _check(tier, layer, topk, meta, out, bt):
    """Every kept key's hot row equals its host row; rejected keys are -1; the residency maps agree."""
    topk, out = topk.cpu(), out.cpu()
    cold = tier.cold[layer].view(-1, ROW).cpu()
    hot = tier.hot[layer].view(-1, ROW).cpu()
    qs, seq, slots = meta.q_start.cpu(), meta.seq_lens.cpu(), meta.state_slots.cpu()
    btc = bt.cpu()
    for b in range(len(seq)):
        for t in range(int(qs[b]), int(qs[b + 1])):
            qpos = int(seq[b]) - (int(qs[b + 1]) - int(qs[b])) + (t - int(qs[b]))
            for e in range(topk.shape[1]):
                p, h = int(topk[t, e]), int(out[t, e])
                if p < 0 or p > qpos:
                    assert h == -1
                    continue
                assert 0 <= h < tier.H
                crow = int(btc[b, p // 64]) * 64 + p % 64
                assert torch.equal(hot[int(slots[b]) * tier.H + h], cold[crow]), (b, t, p, h)
    s2p = tier.slot2pos[layer].cpu()
    p2s = tier.pos2slot[layer].cpu()
    for s in slots.tolist():
        for h, p in enumerate(s2p[s].tolist()):
            if p >= 0:
                assert int(p2s[s, p]) == h
        res = (p2s[s] >= 0).nonzero().flatten().tolist()
        assert all(int(s2p[s, int(p2s[s, p])]) == p for p in res)


def test_resolve_many_steps_matches_host_rows():
    gen = torch.Generator().manual_seed(1)
    tier = _tier(H=256)
    _fill_cold(tier, gen)
    seqs, qlens, slots = [900, 1500, 300], [2, 3, 1], [2, 5, 1]
    bt = torch.stack([torch.randperm(39, generator=gen)[:24] + 1 for _ in seqs]).int().cuda()
    tier.reset(torch.tensor(slots, device="cuda"))
    layer = tier.layer(0)
    for step in range(12):
        meta = _meta(seqs, qlens, slots, bt)
        T = sum(qlens)
        # keys drift: half from a hot window near the end, half anywhere (forces evictions)
        tk = []
        for b, (s, q) in enumerate(zip(seqs, qlens)):
            for _ in range(q):
                near = torch.randint(max(0, s - 200), s, (32,), generator=gen)
                far = torch.randint(0, s, (32,), generator=gen)
                row = torch.cat([near, far]).int()
                row[torch.randperm(64, generator=gen)[:5]] = -1
                row[0] = s + 5  # beyond the query: never kept
                tk.append(row)
        topk = torch.stack(tk).cuda()
        _, hbt, hseq, out = layer.resolve(topk, meta)
        torch.cuda.synchronize()
        tier.check()
        _check(tier, 0, topk, meta, out, bt)
        assert hseq.cpu().tolist() == [tier.H + q for q in qlens]
        assert hbt.cpu()[1].tolist() == list(range(5 * tier.H // 64, 6 * tier.H // 64))
        seqs = [s + q for s, q in zip(seqs, qlens)]
    hits, fetched = tier.stats.tolist()
    assert hits > 0 and fetched > 0


def test_lru_victims_and_rewrite_invalidation():
    gen = torch.Generator().manual_seed(2)
    tier = _tier(H=128)
    _fill_cold(tier, gen)
    bt = (torch.arange(24, dtype=torch.int32) + 1).view(1, 24).cuda()
    tier.reset(torch.tensor([3], device="cuda"))
    layer = tier.layer(0)
    A, B_, C = torch.arange(0, 64), torch.arange(100, 164), torch.arange(200, 264)

    def step(keys, written=None, seq=1000):
        meta = _meta([seq], [1], [3], bt, written)
        topk = keys.int().view(1, -1).cuda()
        _, _, _, out = layer.resolve(topk, meta)
        torch.cuda.synchronize()
        tier.check()
        _check(tier, 0, topk, meta, out, bt)
        return tier.pos2slot[0, 3].cpu()

    step(A)
    step(B_)  # the 128 rows are full: A (older) and B
    before = tier.stats.clone()
    p2s = step(C)  # C evicts A, the least recently used, not B
    assert bool((p2s[A] == -1).all()) and bool((p2s[B_] >= 0).all()) and bool((p2s[C] >= 0).all())
    assert int((tier.stats - before)[1]) == 64
    before = tier.stats.clone()
    step(B_)  # all hits
    d = (tier.stats - before).tolist()
    assert d == [64, 0]
    # position 120 (resident, in B) is rewritten by this step: its new host bytes must be fetched
    p = 120
    crow = int(bt[0, p // 64]) * 64 + p % 64
    tier.cold[0].view(-1, ROW)[crow] = torch.arange(ROW, dtype=torch.int32).to(torch.uint8).cuda()
    before = tier.stats.clone()
    step(B_, written=[crow], seq=p + 1)
    assert (tier.stats - before).tolist()[1] == 1  # only the rewritten position was fetched again


def test_more_keys_than_hot_rows_is_flagged():
    tier = _tier(H=64)
    bt = (torch.arange(24, dtype=torch.int32) + 1).view(1, 24).cuda()
    tier.reset(torch.tensor([1], device="cuda"))
    meta = _meta([1000], [2], [1], bt)
    topk = torch.stack([torch.arange(0, 64), torch.arange(500, 564)]).int().cuda()  # 128 distinct keys
    tier.layer(0).resolve(topk, meta)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="601"):
        tier.check()


@pytest.mark.parametrize("graphs", [False, True])
def test_engine_with_host_tier_generates_the_same_tokens(graphs):
    from vllm_suffix_hybrid_b200.engine.config import (CacheConfig, EngineConfig, SpecConfig, deepseek_v32_config,
                                                       shrink)
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine

    m = shrink(deepseek_v32_config(), layers=3, hidden=256, vocab=1024)
    m.dsa_topk = 64  # a top-k well below the contexts, and hot rows that cannot hold a whole context
    m.kv_format = "nvfp4"
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, 1024, int(n)) for n in (300, 90, 450)]
    outs = []
    for host in (False, True):
        cfg = EngineConfig(model=m, spec=SpecConfig(method="hybrid", k=3),
                           cache=CacheConfig(max_model_len=1024, host_kv=host, host_kv_hot_rows=320, num_blocks=64),
                           max_num_seqs=4, device="cuda", cuda_graphs=graphs)
        eng = LLMEngine(cfg)
        outs.append(eng.generate(prompts, max_new_tokens=24))
        if host:
            assert eng.host_tier is not None
            eng.host_tier.check()
            assert eng.host_tier.hit_rate() is not None
    assert outs[0] == outs[1]
