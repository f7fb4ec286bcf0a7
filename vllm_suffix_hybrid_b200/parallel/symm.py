"""Symmetric-memory communicator for tensor parallelism over NVLink.

Buffers come from torch's symmetric-memory allocator (one mapping of every
rank's buffer in every process); the data path is this framework's own
kernel (``_C.allreduce_fused``): row-parallel GEMMs write their partial sums
into the local ``partial(T)`` buffer, and one kernel pushes them to the
peers with NVLink stores into double-buffered receive slots, reduces in rank
order and applies the residual add + RMSNorm.

Routing by the bytes each rank sends (the reference routes its all-reduce by
size bands too, reference: suffix_hybrid/nccl_split.py:63-77): one-shot
(push the whole partial to every peer, one cross-GPU wait) while
(world - 1) * T * H * 2 bytes stay under ``one_shot_max_bytes``, two-shot
(reduce-scatter to row owners, all-gather of the sums, two waits) above it.
Every call uses the same grid (all blocks then share one epoch parity).
Device-side waits time out into ``err``; ``check()`` raises on the host if
any collective failed.
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from . import state

MAX_BLOCKS = 160
PHASES = 3
MAX_WORLD = 8


def qar_mode(name: str) -> int:
    """Compressed all-reduce mode of the kernel: 0 off, 1 int8, 2 fp8 e4m3."""
    name = (name or "").strip().lower()
    if name in ("", "0", "off", "none"):
        return 0
    if name not in ("int8", "fp8"):
        raise ValueError(f"SUFFIX_NCCL_QAR must be int8 or fp8, got {name!r}")
    return 1 if name == "int8" else 2


def qar_reference(parts, mode: int, two_shot: bool = False, world_chunks: int = 1) -> torch.Tensor:
    """CPU statement of the compressed all-reduce for a list of per-rank fp32 partials [T, H]: every
    partial is encoded per 128-value block (scale = amax / 127 for int8 or amax / 448 for fp8 e4m3, codes
    round(x / scale) clamped to [-127, 127] or e4m3(x / scale)) and decoded, the decoded rows are summed
    in rank order, and with ``two_shot`` the sum is encoded and decoded once more (the owner's gather)."""

    def roundtrip(x: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        blk = x.float().view(T, H // 128, 128)
        amax = blk.abs().amax(-1, keepdim=True)
        qmax = 127.0 if mode == 1 else 448.0
        scale = amax / qmax
        inv = torch.where(amax > 0, qmax / amax, torch.zeros_like(amax))
        if mode == 1:
            codes = torch.clamp(torch.round(blk * inv), -127, 127)
        else:
            codes = torch.clamp(blk * inv, -448, 448).to(torch.float8_e4m3fn).float()
        return (codes * scale).view(T, H)

    acc = torch.zeros_like(parts[0], dtype=torch.float32)
    for x in parts:
        acc = acc + roundtrip(x)
    return roundtrip(acc) if two_shot else acc


class SymmComm:
    def __init__(self, hidden: int, max_tokens: int, dtype=torch.bfloat16, group=None,
                 one_shot_max_bytes: Optional[int] = None):
        import torch.distributed._symmetric_memory as symm_mem

        st = state.get()
        self.rank, self.world = st.rank, st.world
        if self.world > MAX_WORLD:
            raise ValueError(f"fused NVLink collectives support up to {MAX_WORLD} ranks")
        self.group = group or st.group
        self.hidden, self.max_tokens = hidden, max_tokens
        dev = torch.device("cuda", torch.cuda.current_device())
        self.partial_buf = torch.empty(max_tokens, hidden, dtype=dtype, device=dev)
        self.recv_buf = symm_mem.empty(2 * self.world * max_tokens * hidden, dtype=dtype, device=dev)
        self.gather_buf = symm_mem.empty(2 * max_tokens * hidden, dtype=dtype, device=dev)
        self.gather_res_buf = symm_mem.empty(2 * max_tokens * hidden, dtype=dtype, device=dev)
        # flags [PHASES][MAX_BLOCKS][MAX_WORLD] then the reduce-scatter arrival counters [2]
        self.flag_buf = symm_mem.empty(PHASES * MAX_BLOCKS * MAX_WORLD + 64, dtype=torch.int32, device=dev)
        self.flag_buf.zero_()
        torch.cuda.synchronize()
        name = self.group.group_name if hasattr(self.group, "group_name") else dist.group.WORLD.group_name
        h_r = symm_mem.rendezvous(self.recv_buf, name)
        h_g = symm_mem.rendezvous(self.gather_buf, name)
        h_f = symm_mem.rendezvous(self.flag_buf, name)
        h_gr = symm_mem.rendezvous(self.gather_res_buf, name)
        self.peer_recv = [int(x) for x in h_r.buffer_ptrs]
        self.peer_gather = [int(x) for x in h_g.buffer_ptrs]
        self.peer_gather_res = [int(x) for x in h_gr.buffer_ptrs]
        self.peer_flags = [int(x) for x in h_f.buffer_ptrs]
        cnt_off = PHASES * MAX_BLOCKS * MAX_WORLD * 4
        self.peer_rs_cnt = [p + cnt_off for p in self.peer_flags]
        # Vocab-parallel argmax: keys [2][world][max_tokens] (u64) then flags [MAX_BLOCKS][MAX_WORLD] (u32).
        self.key_words = 2 * self.world * max_tokens
        self.argmax_buf = symm_mem.empty(self.key_words * 2 + MAX_BLOCKS * MAX_WORLD, dtype=torch.int32, device=dev)
        self.argmax_buf.zero_()
        torch.cuda.synchronize()
        h_a = symm_mem.rendezvous(self.argmax_buf, name)
        self.peer_keys = [int(x) for x in h_a.buffer_ptrs]
        self.peer_argmax_flags = [p + self.key_words * 8 for p in self.peer_keys]
        self.argmax_counters = torch.zeros(MAX_BLOCKS, dtype=torch.int32, device=dev)
        self.argmax_blocks = min(MAX_BLOCKS, 64)
        self._handles = (h_r, h_g, h_f, h_gr, h_a)
        self.targets = torch.zeros(2 * MAX_BLOCKS, dtype=torch.int32, device=dev)
        # Row-parallel GEMMs push their rows straight to the owners (reduce-scatter in
        # the GEMM epilogue) and rs_norm_ag finishes; SH_TP_PUSH=0 keeps the
        # GEMM -> all-reduce kernel path.
        self.push_enabled = os.environ.get("SH_TP_PUSH", "1") != "0"
        self.counters = torch.zeros(MAX_BLOCKS, dtype=torch.int32, device=dev)
        self.timing = None  # set to an int64 [64, 4] tensor to record per-call phase stamps
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.blocks = min(MAX_BLOCKS, sms)
        env = os.environ.get("SH_ONE_SHOT_MAX_BYTES")
        self.one_shot_max_bytes = int(env) if env else (one_shot_max_bytes or (4 << 20))
        # L2 prefetch of the next GEMM's weights from the collective kernels (SH_L2_PREFETCH_MAX_BYTES=0: off)
        self.l2_prefetch_max_bytes = int(os.environ.get("SH_L2_PREFETCH_MAX_BYTES", str(24 << 20)))
        # Compressed all-reduce (off by default; lossy): SUFFIX_NCCL_QAR=int8|fp8 sends every partial as
        # 1-byte codes + one fp32 scale per 128 values for bf16 messages of SUFFIX_NCCL_QAR_MIN_BYTES
        # (4 MiB) up to SUFFIX_NCCL_QAR_MAX_BYTES (no limit) -- the reference's knobs and band (reference:
        # suffix_hybrid/nccl_split.py:37-39, suffix_hybrid/nccl_qar.py:1-25).
        self.qar_mode = qar_mode(os.environ.get("SUFFIX_NCCL_QAR", ""))
        self.qar_min_bytes = int(os.environ.get("SUFFIX_NCCL_QAR_MIN_BYTES", str(4 << 20)))
        self.qar_max_bytes = int(os.environ.get("SUFFIX_NCCL_QAR_MAX_BYTES", str(1 << 62)))
        dist.barrier(group=self.group)

    # -- buffers --------------------------------------------------------------
    def partial(self, tokens: int) -> torch.Tensor:
        """The [tokens, hidden] slice a row-parallel GEMM writes its partial into."""
        if tokens > self.max_tokens:
            raise ValueError(f"{tokens} tokens exceed the symmetric buffer ({self.max_tokens})")
        return self.partial_buf[:tokens]

    def owns(self, x: torch.Tensor) -> bool:
        return x.data_ptr() == self.partial_buf.data_ptr() and x.shape[-1] == self.hidden

    def can_all_reduce(self, x: torch.Tensor) -> bool:
        return self.owns(x) and x.shape[0] <= self.max_tokens

    # -- collectives ----------------------------------------------------------
    def _prefetch(self, nxt: Optional[torch.Tensor]):
        """(pointer, bytes) of the next GEMM's weight to pull into L2 while the ranks wait (C7: the
        reference prefetches the next window's weights from its waiting all-reduce blocks, reference:
        suffix_hybrid/host_ar.py:106-127).  Capped at ``l2_prefetch_max_bytes`` (the head of the weight,
        which the GEMM's first tile wave reads)."""
        if nxt is None or not self.l2_prefetch_max_bytes:
            return 0, 0
        return nxt.data_ptr(), min(nxt.numel() * nxt.element_size(), self.l2_prefetch_max_bytes)

    def _launch(self, x: torch.Tensor, out: torch.Tensor, residual=None, weight=None, eps: float = 0.0,
                prefetch: Optional[torch.Tensor] = None) -> None:
        from .. import ops

        T, H = x.shape
        sent = (self.world - 1) * T * H * x.element_size()
        two_shot = sent > self.one_shot_max_bytes and T >= self.world
        pf, pf_bytes = self._prefetch(prefetch)
        msg = T * H * x.element_size()
        quant = self.qar_mode if (self.qar_mode and H % 128 == 0 and
                                  self.qar_min_bytes <= msg < self.qar_max_bytes) else 0
        ops.native().allreduce_fused(x, self.peer_recv, self.peer_gather, self.peer_flags, self.counters, out,
                                     residual, weight, self.err, self.rank, T, H, self.max_tokens, eps, two_shot,
                                     self.blocks, self.timing, pf, pf_bytes, quant)

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(x)
        self._launch(x, out)
        return out

    def all_reduce_add_rms_norm(self, x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor,
                                eps: float, prefetch: Optional[torch.Tensor] = None) -> torch.Tensor:
        out = torch.empty_like(x)
        self._launch(x, out, residual, w, eps, prefetch)
        return out

    # -- reduce-scatter in the GEMM epilogue -----------------------------------
    def owner_rows(self, T: int) -> int:
        return max(1, -(-T // self.world))

    def push_expected(self, T: int, N: int, swap: bool, bn: int) -> int:
        """Arrival counts this rank receives for one push GEMM (mirrors the epilogue's per-warp counting)."""
        Tc = self.owner_rows(T)
        lo, hi = self.rank * Tc, min(T, (self.rank + 1) * Tc)
        if lo >= hi:
            return 0
        if swap:  # every warp of every (weight tile, token tile) counts the tile's token range
            tiles_w = -(-N // 128)
            n = sum(1 for t0 in range(0, T, bn) if t0 < hi and min(t0 + bn, T) > lo)
            return self.world * tiles_w * 4 * n
        tiles_w = -(-N // bn)  # every warp counts its own 32 token rows
        n = sum(1 for r0 in range(0, T, 32) if r0 < hi and min(r0 + 32, T) > lo)
        return self.world * tiles_w * n

    def push_gemm(self, x: torch.Tensor, w: torch.Tensor) -> "PushedPartial":
        """Row-parallel y = x w^T with the rows pushed to their owner ranks; finish with finish_push()."""
        from .. import ops

        T, N = x.shape[0], w.shape[0]
        if N != self.hidden or T > self.max_tokens:
            raise ValueError("push GEMM: output width must be the hidden size and T <= max_tokens")
        from ..ops import gemm

        x = x.contiguous()
        # The push epilogue writes 128-byte token-row segments: tokens on the MMA M side (no swap),
        # no split-K.  The tile configuration is autotuned on the same GEMM with a local epilogue.
        pair, bn = gemm.plan_push(x, w)
        ops.native().gemm_bf16_push(x, w, pair, bn, self.peer_recv, self.peer_rs_cnt, self.counters, self.rank,
                                    self.owner_rows(T), self.max_tokens, self.err)
        return PushedPartial(self, T, self.push_expected(T, N, False, bn))

    def finish_push(self, pp: "PushedPartial", residual: torch.Tensor, w: torch.Tensor, eps: float,
                    gather_residual: bool = False, prefetch: Optional[torch.Tensor] = None) -> torch.Tensor:
        from .. import ops

        out = torch.empty(pp.T, self.hidden, dtype=residual.dtype, device=residual.device)
        pf, pf_bytes = self._prefetch(prefetch)
        ops.native().rs_norm_ag(self.peer_recv[self.rank], self.peer_gather, self.peer_gather_res, self.peer_flags,
                                self.peer_rs_cnt[self.rank], self.targets, self.counters, residual, out, w, self.err,
                                self.rank, pp.T, self.hidden, self.max_tokens, self.owner_rows(pp.T), pp.expected,
                                eps, gather_residual, self.blocks, self.timing, pf, pf_bytes)
        return out

    # -- vocab-parallel argmax --------------------------------------------------
    def can_argmax(self, logits: torch.Tensor) -> bool:
        return (logits.is_cuda and logits.dtype == torch.bfloat16 and logits.dim() == 2 and logits.stride(1) == 1
                and logits.shape[0] <= self.max_tokens and (logits.stride(0) * 2) % 16 == 0
                and logits.data_ptr() % 16 == 0)

    def argmax(self, logits: torch.Tensor, vocab_offset: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Global greedy ids of vocab-sharded logits [T, V/tp] in one kernel (keys over NVLink)."""
        from .. import ops

        dst = out if out is not None and out.is_contiguous() and out.dtype == torch.int64 else \
            torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
        ops.native().argmax_tp(dst, logits, self.peer_keys, self.peer_argmax_flags, self.argmax_counters, self.err,
                               self.rank, self.max_tokens, vocab_offset, self.argmax_blocks)
        if out is not None and dst is not out:
            out.copy_(dst)
            return out
        return dst

    def check(self) -> None:
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"symmetric-memory collective timed out or failed (code {code}) on rank {self.rank}")


class PushedPartial:
    """A row-parallel GEMM output that was pushed to its owner ranks (not materialised locally)."""

    def __init__(self, comm: SymmComm, T: int, expected: int):
        self.comm, self.T, self.expected = comm, T, expected
        self.shape = (T, comm.hidden)
