"""Failure detection of the cross-rank kernels, without a GPU fault.

Every cross-GPU wait in the NVLink collectives and the expert-parallel
all-to-all is bounded: when the peer's flag does not arrive in time the
kernel records an error code in its `err` word and returns, and the host
sees the code (``SymmComm.check()`` raises).  These tests make a wait run
out on ONE GPU: the kernels run in a two-rank layout whose "peer" buffers
are plain allocations on this GPU that nobody writes, with the wait limit
shortened to 1 ms.  Nothing traps, hangs or faults; after the failed call
the context is still usable and a call whose peer flag is present passes.
"""
import pytest
import torch

from vllm_suffix_hybrid_b200 import ops

pytestmark = pytest.mark.gpu

MAX_BLOCKS, MAX_WORLD, PHASES = 160, 8, 3
WAIT_NS = 1_000_000  # 1 ms


@pytest.fixture
def short_waits():
    lib = ops.native()
    old = lib.get_wait_ns()
    lib.set_wait_ns(WAIT_NS)
    yield lib
    lib.set_wait_ns(old)


def _flags():
    return torch.zeros(PHASES * MAX_BLOCKS * MAX_WORLD + 64, dtype=torch.int32, device="cuda")


def test_allreduce_wait_times_out_and_recovers(short_waits):
    from vllm_suffix_hybrid_b200.parallel.symm import SymmComm

    lib = short_waits
    torch.manual_seed(0)
    T, H, max_T, blocks = 5, 256, 8, 4
    recv = [torch.zeros(2 * 2 * max_T * H, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    gather = [torch.zeros(2 * max_T * H, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    flags = [_flags(), _flags()]
    counters = torch.zeros(MAX_BLOCKS, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    partial = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    out = torch.full((T, H), float("nan"), dtype=torch.bfloat16, device="cuda")
    ptrs = lambda xs: [x.data_ptr() for x in xs]  # noqa: E731

    # Rank 0 of a two-rank one-shot all-reduce: rank 1's flag never arrives.
    lib.allreduce_fused(partial, ptrs(recv), ptrs(gather), ptrs(flags), counters, out, None, None, err, 0, T, H,
                        max_T, 0.0, False, blocks)
    torch.cuda.synchronize()  # the kernel returned
    assert int(err.item()) == 100  # phase 0 wait expired
    assert bool(torch.isnan(out.float()).all())  # no result was written past the failed wait
    comm = SymmComm.__new__(SymmComm)
    comm.err, comm.rank = err, 0
    with pytest.raises(RuntimeError, match="code 100"):
        comm.check()

    # Next call (epoch 2, parity 0): play rank 1 -- its rows in our receive slot, its flags raised.
    err.zero_()
    other = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    recv[0].view(2, 2, max_T, H)[0, 1, :T] = other
    fl = flags[0].view(-1)[: PHASES * MAX_BLOCKS * MAX_WORLD].view(PHASES, MAX_BLOCKS, MAX_WORLD)
    fl[0, :blocks, 1] = 2
    lib.allreduce_fused(partial, ptrs(recv), ptrs(gather), ptrs(flags), counters, out, None, None, err, 0, T, H,
                        max_T, 0.0, False, blocks)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want = (partial.float() + other.float()).to(torch.bfloat16)
    assert torch.equal(out, want)
    comm.check()


def test_argmax_wait_times_out(short_waits):
    lib = short_waits
    T, V, max_T = 6, 1024, 8
    logits = torch.randn(T, V, device="cuda").to(torch.bfloat16)
    bufs = [torch.zeros(2 * 2 * max_T * 2 + MAX_BLOCKS * MAX_WORLD, dtype=torch.int32, device="cuda")
            for _ in range(2)]
    keys = [b.data_ptr() for b in bufs]
    flags = [k + 2 * 2 * max_T * 8 for k in keys]
    counters = torch.zeros(MAX_BLOCKS, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.full((T,), -7, dtype=torch.int64, device="cuda")
    lib.argmax_tp(out, logits, keys, flags, counters, err, 0, max_T, 0, 8)
    torch.cuda.synchronize()
    assert int(err.item()) == 100
    assert bool((out == -7).all())


def test_ep_dispatch_wait_times_out(short_waits):
    lib = short_waits
    T, H, k, e_local, max_T, blocks = 4, 256, 2, 4, 8, 4
    world = 2
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    ids = torch.tensor([[0, 5], [1, 6], [2, 3], [7, 4]], dtype=torch.int32, device="cuda")
    w = torch.full((T, k), 0.5, device="cuda")
    mk = lambda shape, dt: [torch.zeros(shape, dtype=dt, device="cuda") for _ in range(world)]  # noqa: E731
    px = mk((world * max_T, H), torch.bfloat16)
    pid = mk((world * max_T, k), torch.int32)
    pw = mk((world * max_T, k), torch.float32)
    py = mk((world * max_T, H), torch.bfloat16)
    pf = mk((2 * MAX_BLOCKS * MAX_WORLD,), torch.int32)
    ptrs = lambda xs: [t.data_ptr() for t in xs]  # noqa: E731
    counters = torch.zeros(MAX_BLOCKS, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    lib.ep_dispatch(x, ids, w, ptrs(px), ptrs(pid), ptrs(pw), ptrs(py), ptrs(pf), counters, err, 0, e_local, max_T,
                    blocks, [], [], [], None, None, False, 1, 1, False, 1.0)
    torch.cuda.synchronize()
    assert int(err.item()) == 200  # the dispatch barrier (phase 0) expired
    # This rank's own rows still reached the ranks that host their experts (here: both "peers").
    assert torch.equal(px[0][0], x[0]) and torch.equal(px[1][3], x[3])
