"""Host KV tier (HiSparse) for DSA sparse-attention models.

The full MLA latent cache lives in pinned host memory mapped into the GPU's address space; the GPU keeps
only `hot_rows` rows per request slot and layer.  Every decode step, after the DSA indexer has chosen each
query token's top-k keys, `csrc/kernels/hisparse.cu` resolves the keys against the request's hot rows
(hits stay, misses are fetched from host memory into least-recently-used rows) and rewrites the top-k list
as hot-row indices, so the MLA kernel reads a small device cache whose rows are byte-identical to the host
cache's.  Prefill reads and writes the host cache directly; decode writes its new rows there and drops the
hot copy of every rewritten position.

This lets the number of long requests grow with host memory instead of HBM: the device holds the indexer
keys (132 B per token) and `slots x hot_rows` latent rows per layer, the host the 352-byte (NVFP4) or
1152-byte (bf16) latent rows of every token.

Reference parity: the HiSparse hot buffer over a host-pinned KV pool and its device resolver (reference:
sm120/hisparse_mtp_patch/own_resolver.py:200-690, host pool sitecustomize.py:574-581).
"""
from __future__ import annotations

from typing import List, Optional

import torch

MAX_HOT_ROWS = 16384


def hot_rows_for(k: int, topk: int) -> int:
    """Default hot rows per request and layer: every key one verify step can select ((k + 1) x top-k
    distinct keys at most) plus one top-k of slack for reuse across steps, in 64-row blocks."""
    need = (k + 2) * topk
    return int(min(MAX_HOT_ROWS, -(-need // 64) * 64))


def resolve_reference(pos2slot, slot2pos, stamp, tick: int, topk, qpos, written=()):
    """CPU statement of one request's resolve, the policy of `csrc/kernels/hisparse.cu` (numpy int arrays of
    one request slot, updated in place).

    topk [T, K] key positions of the request's T query tokens (-1: none), qpos [T] their positions, written
    the positions the step writes.  Returns (hot [T, K] hot-row indices or -1, hits, fetched positions in
    claim order, overflow).  Victims are the rows no key of this step uses, free rows first, then by age
    (tick - stamp) capped at 255 steps, oldest first; the kernel takes rows of the threshold age in any
    order, this statement by row index."""
    import numpy as np

    H = slot2pos.shape[0]
    for p in written:  # rewritten positions lose their hot copy
        if 0 <= p < pos2slot.shape[0] and pos2slot[p] >= 0:
            slot2pos[pos2slot[p]] = -1
            pos2slot[p] = -1
    topk = np.asarray(topk)
    valid = (topk >= 0) & (topk <= np.asarray(qpos)[:, None]) & (topk < pos2slot.shape[0])
    hits, miss = 0, []
    claimed = set()
    for p in topk[valid].tolist():
        h = pos2slot[p]
        if h >= 0:
            stamp[h] = tick
            hits += 1
        elif p not in claimed:
            claimed.add(p)
            miss.append(p)
    used = (slot2pos >= 0) & (stamp == tick)
    age = np.where(slot2pos < 0, 255, np.clip(tick - stamp, 1, 255))
    order = [h for h in sorted(range(H), key=lambda h: (-int(age[h]), h)) if not used[h]]
    overflow = len(miss) > len(order)
    fetched = []
    for p, h in zip(miss, order):
        if slot2pos[h] >= 0:
            pos2slot[slot2pos[h]] = -1
        slot2pos[h], stamp[h], pos2slot[p] = p, tick, h
        fetched.append(p)
    out = np.full(topk.shape, -1, dtype=np.int64)
    out[valid] = np.maximum(pos2slot[topk[valid]], -1)
    return out, hits, fetched, overflow


class HostTierLayer:
    """One layer's view of the tier: its host cache, hot rows, residency maps and resolve outputs."""

    def __init__(self, tier: "HostKVTier", i: int):
        self.tier, self.i = tier, i
        self.cold = tier.cold[i]
        self.hot = tier.hot[i]

    def resolve(self, topk: torch.Tensor, meta):
        """Top-k positions [T, K] -> (hot cache, hot block tables [B, H/64], lengths [B], hot top-k [T, K])."""
        t = self.tier
        T, B = topk.shape[0], meta.seq_lens.shape[0]
        out = t.topk_out[:T, : topk.shape[1]]
        t.lib.hisparse_resolve(topk, out, meta.q_start, meta.seq_lens, meta.state_slots, meta.positions,
                               meta.slot_mapping, meta.block_tables, self.cold, self.hot, t.pos2slot[self.i],
                               t.slot2pos[self.i], t.stamp[self.i], t.clock[self.i], t.hot_bt[:B], t.hot_seq[:B],
                               t.err, t.stats)
        return self.hot, t.hot_bt[:B], t.hot_seq[:B], out


class HostKVTier:
    """Host-resident latent caches of `layers` layers plus their device hot rows and residency maps."""

    def __init__(self, layers: int, num_blocks: int, block_size: int, row_shape: tuple, dtype: torch.dtype,
                 slots: int, hot_rows: int, max_positions: int, max_tokens: int, max_topk: int, device):
        if block_size != 64:
            raise ValueError("the host KV tier uses 64-token blocks")
        if hot_rows % 64 or not 0 < hot_rows <= MAX_HOT_ROWS:
            raise ValueError(f"hot_rows must be a multiple of 64 in (0, {MAX_HOT_ROWS}], got {hot_rows}")
        from .. import ops

        self.lib = ops.native()
        self.layers, self.slots, self.H = layers, slots, hot_rows
        self.P = -(-max_positions // 64) * 64
        elem = torch.empty(0, dtype=dtype).element_size()
        row_elems = 1
        for d in row_shape:
            row_elems *= d
        self.row_bytes = row_elems * elem
        per_layer = num_blocks * block_size * self.row_bytes
        self.cold: List[torch.Tensor] = []
        for _ in range(layers):
            buf = self.lib.mapped_host_buffer(per_layer)
            self.cold.append(buf.view(dtype).view(num_blocks, block_size, *row_shape))
        hb = slots * hot_rows // 64
        self.hot = [torch.zeros(hb, 64, *row_shape, dtype=dtype, device=device) for _ in range(layers)]
        self.pos2slot = torch.full((layers, slots, self.P), -1, dtype=torch.int32, device=device)
        self.slot2pos = torch.full((layers, slots, hot_rows), -1, dtype=torch.int32, device=device)
        self.stamp = torch.zeros((layers, slots, hot_rows), dtype=torch.int32, device=device)
        self.clock = torch.zeros((layers, slots), dtype=torch.int32, device=device)
        self.topk_out = torch.full((max_tokens, max_topk), -1, dtype=torch.int32, device=device)
        self.hot_bt = torch.zeros((slots, hot_rows // 64), dtype=torch.int32, device=device)
        self.hot_seq = torch.zeros(slots, dtype=torch.int64, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.stats = torch.zeros(2, dtype=torch.int64, device=device)  # hits, rows fetched from the host
        self.host_bytes = per_layer * layers
        self.device_bytes = (hb * 64 * self.row_bytes + (slots * self.P + 2 * slots * hot_rows) * 4) * layers

    def layer(self, i: int) -> HostTierLayer:
        return HostTierLayer(self, i)

    def reset(self, state_slots: torch.Tensor) -> None:
        """Forget the residency of request slots that new requests take (all layers)."""
        self.lib.hisparse_reset(self.pos2slot, self.slot2pos, self.stamp, self.clock, state_slots)

    def check(self) -> None:
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"host KV tier: error {code} (601: more distinct keys in one step than hot rows)")

    def hit_rate(self) -> Optional[float]:
        hits, fetched = (int(x) for x in self.stats.tolist())
        return hits / (hits + fetched) if hits + fetched else None
