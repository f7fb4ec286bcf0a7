"""The allocation-free attention entry point, called through its C symbol.

`sh_paged_attention_noalloc` serves callers that cannot allocate device
memory where they run attention (for example a C or Rust host runtime that
links only this library and has no device allocator of its own, or a fixed,
pre-reserved memory budget).  It keeps its split-KV partials in a fixed
device array inside the library.  This test loads the exported symbol with
ctypes, runs it twice in a row, and checks each result against the regular
entry point (which takes caller-provided workspaces) on the same inputs.
The file name sorts last so a run stopping at the first failure has already
run every other test; it also passes alone in a fresh process.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ERR_ARGS = -101
ERR_TOO_LARGE = -102


class AttnParams(ctypes.Structure):
    _fields_ = [
        ("out", ctypes.c_void_p), ("out_stride", ctypes.c_int64),
        ("q", ctypes.c_void_p), ("q_stride", ctypes.c_int64),
        ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
        ("block_tables", ctypes.c_void_p), ("bt_stride", ctypes.c_int64),
        ("seq_lens", ctypes.c_void_p), ("q_start", ctypes.c_void_p),
        ("tile_req", ctypes.c_void_p), ("tile_row0", ctypes.c_void_p),
        ("part_o", ctypes.c_void_p), ("part_ml", ctypes.c_void_p), ("err", ctypes.c_void_p),
        ("num_tokens", ctypes.c_int64),
        ("hq", ctypes.c_int), ("hk", ctypes.c_int), ("nsplit", ctypes.c_int), ("scale_log2", ctypes.c_float),
    ]


def _lib():
    import vllm_suffix_hybrid_b200._C as ext

    lib = ctypes.CDLL(ext.__file__)
    fn = lib.sh_paged_attention_noalloc
    fn.argtypes = [ctypes.POINTER(AttnParams), ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p]
    fn.restype = ctypes.c_int
    cap = lib.sh_paged_attention_noalloc_capacity
    cap.restype = ctypes.c_int64
    return fn, cap()


def _case(seed, q_lens=(6, 6, 6, 1), ctx=(300, 64, 1000, 2047)):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q_lens, ctx = list(q_lens), list(ctx)
    hq, hk, d, bs = 8, 2, 128, 64
    seq = [c + q for c, q in zip(ctx, q_lens)]
    maxb = max((s + bs - 1) // bs for s in seq)
    nblocks = len(q_lens) * maxb + 1
    kc = torch.randn(nblocks, hk, bs, d, generator=g).to("cuda", torch.bfloat16)
    vc = torch.randn(nblocks, hk, bs, d, generator=g).to("cuda", torch.bfloat16)
    bt = (torch.randperm(nblocks - 1, generator=g)[: len(q_lens) * maxb] + 1).view(len(q_lens), maxb)
    T = sum(q_lens)
    qkv = torch.randn(T, (hq + 2 * hk) * d, generator=g).to("cuda", torch.bfloat16)
    tr, t0 = [], []
    for b, ql in enumerate(q_lens):
        for r in range(0, ql * (hq // hk), 64):
            tr.append(b)
            t0.append(r)
    return dict(qkv=qkv, kc=kc, vc=vc, bt=bt.int().cuda(), seq=torch.tensor(seq, device="cuda"),
                qs=torch.tensor([0] + list(np.cumsum(q_lens)), device="cuda"),
                tr=torch.tensor(tr, dtype=torch.int32, device="cuda"),
                t0=torch.tensor(t0, dtype=torch.int32, device="cuda"), hq=hq, hk=hk, d=d, T=T,
                max_rows=min(64, max(q_lens) * (hq // hk)))


def _params(c, out, nsplit):
    return AttnParams(
        out=out.data_ptr(), out_stride=out.stride(0), q=c["qkv"].data_ptr(), q_stride=c["qkv"].stride(0),
        k_cache=c["kc"].data_ptr(), v_cache=c["vc"].data_ptr(), block_tables=c["bt"].data_ptr(),
        bt_stride=c["bt"].stride(0), seq_lens=c["seq"].data_ptr(), q_start=c["qs"].data_ptr(),
        tile_req=c["tr"].data_ptr(), tile_row0=c["t0"].data_ptr(), part_o=None, part_ml=None, err=None,
        num_tokens=c["T"], hq=c["hq"], hk=c["hk"], nsplit=nsplit,
        scale_log2=(1.0 / math.sqrt(c["d"])) * 1.4426950408889634)


def test_noalloc_matches_workspace_entry_point_twice():
    from vllm_suffix_hybrid_b200 import ops

    torch.cuda.set_device(0)
    fn, capacity = _lib()
    nsplit = 4
    stream = torch.cuda.current_stream().cuda_stream
    # Two calls in a row.  The second is smaller (fewer tokens, shorter
    # contexts), so partials left in the shared array by the first call
    # would change its result if the merge ever read a slot it did not write.
    for seed, q_lens, ctx in ((1, (6, 6, 6, 1), (300, 64, 1000, 2047)), (2, (6, 1), (130, 700))):
        c = _case(seed, q_lens, ctx)
        want = torch.empty(c["T"], c["hq"] * c["d"], device="cuda", dtype=torch.bfloat16)
        ops.paged_attention(want, c["qkv"], c["kc"], c["vc"], c["bt"], c["seq"], c["qs"], c["tr"], c["t0"], c["hq"],
                            1.0 / math.sqrt(c["d"]), nsplit, c["max_rows"])
        got = torch.full_like(want, float("nan"))
        torch.cuda.synchronize()
        before = torch.cuda.memory_allocated()
        p = _params(c, got, nsplit)
        rc = fn(ctypes.byref(p), c["tr"].numel(), c["kc"].shape[0], c["d"], c["max_rows"], stream)
        torch.cuda.synchronize()
        assert rc == 0, rc
        assert torch.cuda.memory_allocated() == before  # torch's allocator saw nothing
        assert c["T"] * c["hq"] * nsplit * (c["d"] + 2) <= capacity
        # Same kernels and split order as the workspace entry point: the
        # results must agree bit for bit.
        assert torch.equal(got, want), (got.float() - want.float()).abs().max().item()


def test_noalloc_rejects_oversized_request():
    torch.cuda.set_device(0)
    fn, capacity = _lib()
    c = _case(3)
    out = torch.empty(c["T"], c["hq"] * c["d"], device="cuda", dtype=torch.bfloat16)
    p = _params(c, out, 4)
    p.num_tokens = capacity  # far beyond the fixed scratch
    rc = fn(ctypes.byref(p), c["tr"].numel(), c["kc"].shape[0], c["d"], c["max_rows"],
            torch.cuda.current_stream().cuda_stream)
    assert rc == ERR_TOO_LARGE


def test_noalloc_rejects_bad_sizes_before_any_launch():
    torch.cuda.set_device(0)
    fn, _ = _lib()
    c = _case(4)
    out = torch.empty(c["T"], c["hq"] * c["d"], device="cuda", dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    for tokens, want in ((2 ** 62, ERR_TOO_LARGE), (2 ** 63 - 1, ERR_TOO_LARGE), (-1, ERR_ARGS)):
        p = _params(c, out, 4)
        p.num_tokens = tokens  # a product of this with the other sizes would overflow int64
        rc = fn(ctypes.byref(p), c["tr"].numel(), c["kc"].shape[0], c["d"], c["max_rows"], stream)
        assert rc == want, (tokens, rc)
