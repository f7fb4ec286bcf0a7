"""Expert-parallel all-to-all over NVLink peer memory (data-parallel attention + EP).

Every rank holds its own T tokens (the engine pads every rank to the same T per call) and its E/N
experts.  One MoE call:

1. ``ep_dispatch`` (csrc/kernels/ep_a2a.cu): each token row is stored into the receive buffer of
   every rank that hosts one of its top-k experts (P2P stores from the kernel), with a route row
   (local expert ids, -1 for experts elsewhere) on every rank.  For NVFP4 (W4A4) experts the row is
   quantised once in the dispatch kernel and sent as e2m1 codes + e4m3 scales + 1 / g (3.55x fewer
   bytes); the receiving expert GEMMs gather the codes straight into their operand layout.  With
   ``dispatch_routed`` the kernel also runs the router top-k of each token from its logits;
2. this rank's grouped expert GEMMs over the received ``[world*T, H]`` rows;
3. ``ep_combine``: the expert outputs go back to the token owners, which sum them in rank order.  By
   default the experts' weighted per-token sum (``ep_combine_push``) stores its rows straight into the
   owners' return rows, and the owners only meet and sum (``ep_combine_sum``).

This replaces the NCCL all-gather of every token to every rank + reduce-scatter of the partials
(``parallel/ep.py`` ``dp_dispatch_combine`` with ``SH_EP_A2A=0``): a row crosses NVLink only to the
ranks that serve it.  The reference's EP has no all-to-all at all (every rank sees every token,
one all-reduce combines; reference: suffix_hybrid/kernels/nvfp4_moe.py:449-457,
docs/dsv41-comms.md:54-58); this is the device-initiated dispatch / combine of the data-parallel
attention layout (configs 3 / 4: attention DP=8 + EP=8).
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
import torch.distributed as dist

from . import state

MAX_BLOCKS = 160
MAX_WORLD = 8


class EpA2A:
    def __init__(self, hidden: int, max_tokens: int, k: int, e_local: int, group=None, quant: bool = False):
        import torch.distributed._symmetric_memory as symm_mem

        st = state.get()
        self.rank, self.world = st.rank, st.world
        if self.world > MAX_WORLD:
            raise ValueError(f"EP all-to-all supports up to {MAX_WORLD} ranks")
        if self.world * k > 512:
            raise ValueError("EP all-to-all: world * top_k must be <= 512")
        self.group = group or st.group
        self.hidden, self.max_tokens, self.k, self.e_local = hidden, max_tokens, k, e_local
        dev = torch.device("cuda", torch.cuda.current_device())
        rows = self.world * max_tokens
        self.x_buf = symm_mem.empty(rows * hidden, dtype=torch.bfloat16, device=dev)
        self.ids_buf = symm_mem.empty(rows * k, dtype=torch.int32, device=dev)
        self.w_buf = symm_mem.empty(rows * k, dtype=torch.float32, device=dev)
        self.y_buf = symm_mem.empty(rows * hidden, dtype=torch.bfloat16, device=dev)
        self.flag_buf = symm_mem.empty(2 * MAX_BLOCKS * MAX_WORLD, dtype=torch.int32, device=dev)
        self.flag_buf.zero_()
        self.ids_buf.fill_(-1)
        # NVFP4 dispatch: codes [rows, H/2], e4m3 scales [rows, H/16], 1 / g [rows]
        self.quant = quant
        if quant:
            if hidden % 256:
                raise ValueError("NVFP4 dispatch needs hidden % 256 == 0")
            self.q_buf = symm_mem.empty(rows * hidden // 2, dtype=torch.uint8, device=dev)
            self.s_buf = symm_mem.empty(rows * hidden // 16, dtype=torch.uint8, device=dev)
            self.a_buf = symm_mem.empty(rows, dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        name = self.group.group_name if hasattr(self.group, "group_name") else dist.group.WORLD.group_name
        bufs = [self.x_buf, self.ids_buf, self.w_buf, self.y_buf, self.flag_buf]
        if quant:
            bufs += [self.q_buf, self.s_buf, self.a_buf]
        hs = [symm_mem.rendezvous(b, name) for b in bufs]
        self._handles = hs
        ptrs = [[int(p) for p in h.buffer_ptrs] for h in hs]
        self.peer_x, self.peer_ids, self.peer_w, self.peer_y, self.peer_flags = ptrs[:5]
        self.peer_q, self.peer_s, self.peer_a = ptrs[5:] if quant else ([], [], [])
        self.counters = torch.zeros(MAX_BLOCKS, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.blocks = min(MAX_BLOCKS, sms)
        dist.barrier(group=self.group)

    def _args(self):
        return (self.peer_x, self.peer_ids, self.peer_w, self.peer_y, self.peer_flags, self.counters, self.err,
                self.rank, self.e_local, self.max_tokens, self.blocks)

    def dispatch(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor):
        """-> (rows, local ids [world*T, k], weights [world*T, k]) received by this rank; rows are bf16
        [world*T, H], or with an NVFP4 communicator (codes [world*T, H/2], scales [world*T, H/16],
        1 / g [world*T])."""
        from .. import ops

        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the EP receive buffers ({self.max_tokens})")
        ids = ids.to(torch.int32).contiguous()
        ops.native().ep_dispatch(x.contiguous(), ids, w.float().contiguous(), *self._args(), self.peer_q,
                                 self.peer_s, self.peer_a, None, None, False, 1, 1, True, 1.0)
        return self._received(T)

    def dispatch_routed(self, x: torch.Tensor, logits: torch.Tensor, sigmoid_grouped: bool = False, bias=None,
                        n_groups: int = 1, topk_groups: int = 1, renorm: bool = True, scale: float = 1.0):
        """Routes the tokens inside the dispatch kernel (the router top-k of ops.moe_route, bit for bit)
        from the router logits [T, E] -> (received rows, local ids, local weights, ids [T, k], weights
        [T, k]); the combine takes the returned ids."""
        from .. import ops

        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the EP receive buffers ({self.max_tokens})")
        ids = torch.empty(T, self.k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, self.k, dtype=torch.float32, device=x.device)
        ops.native().ep_dispatch(x.contiguous(), ids, w, *self._args(), self.peer_q, self.peer_s, self.peer_a,
                                 logits.contiguous(), bias, sigmoid_grouped, n_groups, topk_groups, renorm, scale)
        return self._received(T) + (ids, w)

    def _received(self, T: int):
        n, H = self.world * T, self.hidden
        if self.quant:
            rows = (self.q_buf[: n * H // 2].view(n, H // 2), self.s_buf[: n * H // 16].view(n, H // 16),
                    self.a_buf[:n])
        else:
            rows = self.x_buf[: n * H].view(n, H)
        return rows, self.ids_buf[: n * self.k].view(n, self.k), self.w_buf[: n * self.k].view(n, self.k)

    def combine(self, y: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        """y [world*T, H] expert outputs of the received rows -> [T, H] sums for this rank's tokens."""
        from .. import ops

        T = ids.shape[0]
        out = torch.empty(T, self.hidden, dtype=torch.bfloat16, device=y.device)
        ops.native().ep_combine(y.contiguous(), ids.to(torch.int32).contiguous(), out, *self._args())
        return out

    def combine_push(self, ys: torch.Tensor, sorted_pos: torch.Tensor, w_l: torch.Tensor, ids_l: torch.Tensor,
                     T: int) -> None:
        """The experts' weighted per-token sum of the received rows (ys [pairs, H] per sorted pair), stored
        straight into the owners' return rows; finish with combine_sum."""
        from .. import ops

        ops.native().ep_combine_push(ys, sorted_pos, w_l.contiguous(), ids_l, T, *self._args())

    def combine_sum(self, ids: torch.Tensor) -> torch.Tensor:
        """[T, H] sums of the rows combine_push returned to this rank, in rank order."""
        from .. import ops

        out = torch.empty(ids.shape[0], self.hidden, dtype=torch.bfloat16, device=ids.device)
        ops.native().ep_combine_sum(ids.to(torch.int32).contiguous(), out, *self._args())
        return out

    def check(self) -> None:
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"EP all-to-all timed out or failed (code {code}) on rank {self.rank}")


_comms: Dict[Tuple[int, int, int, int, bool], EpA2A] = {}


def get(hidden: int, max_tokens: int, k: int, e_local: int, quant: bool = False) -> Optional[EpA2A]:
    """The process's EP communicator for these sizes (created on first use; every rank must call)."""
    key = (hidden, max_tokens, k, e_local, quant)
    c = _comms.get(key)
    if c is None:
        c = _comms[key] = EpA2A(hidden, max_tokens, k, e_local, quant=quant)
    return c
