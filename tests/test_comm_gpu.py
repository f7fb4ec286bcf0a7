"""Fused NVLink all-reduce + residual add + RMSNorm on 2+ GPUs.

Each rank writes a random partial into its symmetric buffer; the fused
kernel's one-shot and two-shot paths must match an fp32 reference of
rms_norm(residual + sum of partials) and be bit-identical on every rank.
Skipped on hosts with fewer than two GPUs.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from vllm_suffix_hybrid_b200.parallel import state
    from vllm_suffix_hybrid_b200.parallel.symm import SymmComm

    state.init(tp=world, backend="nccl", timeout_s=60)
    try:
        H, T_max = 4096, 384
        comm = SymmComm(H, T_max)
        results = {}
        # Consecutive calls alternate modes and sizes: exercises the epoch-parity
        # double buffering of the receive / gather slots.
        seq = [("one_shot", 384), ("two_shot", 384), ("one_shot", 6), ("two_shot", 100), ("plain", 64),
               ("two_shot", 384), ("one_shot", 384), ("plain", 300)] * 2
        for i, (mode, T) in enumerate(seq):
            comm.one_shot_max_bytes = 0 if mode == "two_shot" else 1 << 30
            g = torch.Generator(device="cuda").manual_seed(100 + rank + 17 * i)
            part = comm.partial(T)
            part.copy_(torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16))
            gw = torch.Generator(device="cuda").manual_seed(7 + i)
            resid = torch.randn(T, H, device="cuda", generator=gw).to(torch.bfloat16)
            w = torch.randn(H, device="cuda", generator=gw).to(torch.bfloat16)
            full = part.float().clone()
            dist.all_reduce(full)
            r_ref = (resid.float() + full).to(torch.bfloat16).float()
            x_ref = r_ref * torch.rsqrt(r_ref.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
            resid_k = resid.clone()
            if mode == "plain":
                x = comm.all_reduce(part)
                x_ref, err_r = full, 0.0
            else:
                x = comm.all_reduce_add_rms_norm(part, resid_k, w, 1e-5)
            torch.cuda.synchronize()
            comm.check()
            err_x = (x.float() - x_ref).abs().max().item() / (1.0 + x_ref.abs().max().item())
            if mode != "plain":
                err_r = (resid_k.float() - r_ref).abs().max().item()
            gathered = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(gathered, x)
            same = all(torch.equal(gathered[0], t) for t in gathered)
            results[f"{i}:{mode}:{T}"] = (err_x, err_r, same)
        # Fused vocab-parallel argmax: each rank holds a V/world slice; the kernel's global ids must equal
        # the first-occurrence argmax of the full (all-gathered) logits, ties across ranks included.
        V = 16032 * world
        for i, T in enumerate((1, 64, 384, 7, 384)):
            g = torch.Generator(device="cuda").manual_seed(500 + i)
            full_logits = torch.randn(T, V, device="cuda", generator=g).to(torch.bfloat16)
            full_logits[0, 5] = 40.0
            full_logits[0, V - 3] = 40.0  # tie between the first and the last rank's slices
            lo = rank * (V // world)
            local = full_logits[:, lo:lo + V // world].contiguous()
            got = comm.argmax(local, lo)
            want = full_logits.float().argmax(1)
            torch.cuda.synchronize()
            comm.check()
            results[f"argmax{i}:{T}"] = (0.0 if torch.equal(got, want) else 1.0, 0.0, True)
        q.put((rank, results))
    finally:
        torch.cuda.synchronize()
        state.shutdown()


def test_fused_allreduce_rmsnorm_multi_gpu():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs >= 2 GPUs")
    world = min(world, 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, modes in res.items():
        for mode, (ex, er, same) in modes.items():
            assert ex < 0.02 and er < 0.1 and same, (rank, mode, ex, er, same)
