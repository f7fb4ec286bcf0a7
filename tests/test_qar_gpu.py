"""Compressed (int8 / fp8) all-reduce over NVLink peer memory.

`SUFFIX_NCCL_QAR=int8|fp8` makes the fused all-reduce send every partial as
1-byte codes plus one fp32 scale per 128 values.  The kernel's result must
match the CPU statement `symm.qar_reference` (the same encode / decode / sum
order) up to a one-code rounding flip per contribution, stay inside the
quantisation error bound of the exact sum, and be bit-identical on every
rank.  The one-rank tests run on one GPU with plain allocations as the
symmetric buffers; the two-rank test needs two GPUs.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from vllm_suffix_hybrid_b200 import ops
from vllm_suffix_hybrid_b200.parallel.symm import qar_reference

pytestmark = pytest.mark.gpu

MAX_BLOCKS, MAX_WORLD, PHASES = 160, 8, 3


def _block_scales(x: torch.Tensor, qmax: float) -> torch.Tensor:
    T, H = x.shape
    return (x.float().view(T, H // 128, 128).abs().amax(-1, keepdim=True) / qmax).expand(T, H // 128, 128).reshape(T, H)


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("two_shot", [False, True])
@pytest.mark.parametrize("T,H", [(6, 4096), (96, 7168), (384, 2048)])
def test_compressed_allreduce_one_rank_matches_statement(mode, two_shot, T, H):
    lib = ops.native()
    torch.manual_seed(T + H + mode)
    max_T, blocks = 384, 16
    recv = torch.zeros(2 * 1 * max_T * H, dtype=torch.bfloat16, device="cuda")
    gather = torch.zeros(2 * max_T * H, dtype=torch.bfloat16, device="cuda")
    flags = torch.zeros(PHASES * MAX_BLOCKS * MAX_WORLD + 64, dtype=torch.int32, device="cuda")
    counters = torch.zeros(MAX_BLOCKS, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    partial = (torch.randn(T, H, device="cuda") * torch.rand(T, 1, device="cuda") * 4).to(torch.bfloat16)
    partial[0, :128] = 0  # an all-zero block: scale 0, codes 0
    out = torch.full((T, H), float("nan"), dtype=torch.bfloat16, device="cuda")
    for _ in range(2):  # twice: both parities of the receive slots
        lib.allreduce_fused(partial, [recv.data_ptr()], [gather.data_ptr()], [flags.data_ptr()], counters, out, None,
                            None, err, 0, T, H, max_T, 0.0, two_shot, blocks, quant=mode)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        want = qar_reference([partial.float().cpu()], mode, two_shot)
        got = out.float().cpu()
        qmax = 127.0 if mode == 1 else 448.0
        # one code step per rounding (the kernel's reciprocal may differ from torch's in the last bit)
        step = _block_scales(partial.cpu(), qmax) * (2 if two_shot else 1) * (1 if mode == 1 else 32)
        tol = step * 1.01 + want.abs() * 2 ** -8 + 1e-6
        assert bool((got - want).abs().le(tol).all()), (got - want).abs().max().item()
        exact = partial.float().cpu()
        bound = step * 0.5 * (2 if two_shot else 1) + exact.abs() * (2 ** -8 if mode == 1 else 2 ** -3) + tol
        assert bool((got - exact).abs().le(bound + step).all())
        assert bool(torch.isfinite(got).all())


def test_compressed_allreduce_rejects_unblocked_width():
    lib = ops.native()
    T, H, max_T = 4, 200, 8  # 200 is not a multiple of the 128-value block
    buf = torch.zeros(2 * max_T * H, dtype=torch.bfloat16, device="cuda")
    flags = torch.zeros(PHASES * MAX_BLOCKS * MAX_WORLD + 64, dtype=torch.int32, device="cuda")
    counters = torch.zeros(MAX_BLOCKS, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="code -4"):
        lib.allreduce_fused(x, [buf.data_ptr()], [buf.data_ptr()], [flags.data_ptr()], counters, torch.empty_like(x),
                            None, None, err, 0, T, H, max_T, 0.0, False, 4, quant=1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", SUFFIX_NCCL_QAR="int8",
                      SUFFIX_NCCL_QAR_MIN_BYTES="0")
    import torch.distributed as dist

    from vllm_suffix_hybrid_b200.parallel import state
    from vllm_suffix_hybrid_b200.parallel.symm import SymmComm

    state.init(tp=world, backend="nccl", timeout_s=60)
    try:
        H, T_max = 4096, 384
        comm = SymmComm(H, T_max)
        out = {}
        for i, (two_shot, T) in enumerate([(False, 6), (True, 384), (False, 384), (True, 100)]):
            comm.one_shot_max_bytes = 0 if two_shot else 1 << 30
            part = comm.partial(T)
            g = torch.Generator(device="cuda").manual_seed(300 + rank + 13 * i)
            part.copy_(torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16))
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part.clone())
            x = comm.all_reduce(part)
            torch.cuda.synchronize()
            comm.check()
            want = qar_reference([p.float().cpu() for p in parts], 1, two_shot)
            exact = sum(p.float() for p in parts).cpu()
            xs = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(xs, x)
            same = all(torch.equal(xs[0], t) for t in xs)
            scale = max(_block_scales(p.cpu(), 127.0).max().item() for p in parts)
            out[i] = ((x.float().cpu() - want).abs().max().item(), (x.float().cpu() - exact).abs().max().item(),
                      scale, same)
        q.put((rank, out))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_compressed_allreduce_two_ranks():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, out in res.items():
        for i, (err_ref, err_exact, scale, same) in out.items():
            assert same, (rank, i)
            assert err_ref <= 2 * world * scale * 1.01 + 0.05, (rank, i, err_ref)
            assert err_exact <= 2 * world * scale + 0.05, (rank, i, err_exact)
