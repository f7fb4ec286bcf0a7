"""Row-parallel GEMM with the reduce-scatter in its epilogue + rs_norm_ag, on 2+ GPUs.

Each rank holds a K-shard of x and w; the push GEMM stores its output rows into
the owners' receive slots, rs_norm_ag sums them in rank order, adds the
residual, applies RMSNorm and gathers the normalised rows on every rank.  The
result must match an fp32 reference of rms_norm(residual + sum_r x_r w_r^T) and
be bit-identical on every rank; calls alternate sizes (swap-AB and 128-row
epilogues), residual gathering, and plain all-reduce calls in between (shared
epoch parity).  Skipped with fewer than two GPUs.
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
    res = []
    try:
        H, Kt, T_max = 1024, 512 * world, 400
        comm = SymmComm(H, T_max)
        seq = [(384, False), (6, False), ("ar", 64), (100, True), (257, True), (64, False), ("ar", 300),
               (1, True), (384, True)] * 2
        for i, item in enumerate(seq):
            g = torch.Generator(device="cuda").manual_seed(1000 + i)  # same full operands on every rank
            if item[0] == "ar":
                T = item[1]
                part = comm.partial(T)
                part.copy_(torch.randn(T, H, device="cuda", generator=torch.Generator(device="cuda").manual_seed(
                    7 * i + rank)).to(torch.bfloat16))
                full = part.float().clone()
                dist.all_reduce(full)
                y = comm.all_reduce(part)
                torch.cuda.synchronize()
                res.append((i, "ar", (y.float() - full).abs().max().item() / (1 + full.abs().max().item()), True))
                continue
            T, gres = item
            x = (torch.randn(T, Kt, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
            w = (torch.randn(H, Kt, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
            resid0 = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
            nw = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).to(torch.bfloat16)
            k0, k1 = rank * 512, (rank + 1) * 512
            xs, ws = x[:, k0:k1].contiguous(), w[:, k0:k1].contiguous()
            # reference: bf16 per-rank partials (as the GEMM epilogue rounds them), fp32 rank-order sum
            parts = [(x[:, r * 512:(r + 1) * 512].float() @ w[:, r * 512:(r + 1) * 512].float().t())
                     .to(torch.bfloat16).float() for r in range(world)]
            tot = sum(parts)
            r_ref = (resid0.float() + tot).to(torch.bfloat16).float()
            y_ref = r_ref * torch.rsqrt(r_ref.pow(2).mean(-1, keepdim=True) + 1e-5) * nw.float()
            resid = resid0.clone()
            pp = comm.push_gemm(xs, ws)
            y = comm.finish_push(pp, resid, nw, 1e-5, gather_residual=gres)
            torch.cuda.synchronize()
            comm.check()
            err_y = (y.float() - y_ref).abs().max().item()
            Tc = comm.owner_rows(T)
            own = slice(rank * Tc, min(T, (rank + 1) * Tc))
            rows = slice(0, T) if gres else own
            err_r = (resid[rows].float() - r_ref[rows]).abs().max().item() if T > rank * Tc else 0.0
            gathered = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(gathered, y)
            same = all(torch.equal(gathered[0], t) for t in gathered)
            res.append((i, T, max(err_y, err_r), same))
        q.put((rank, res))
    finally:
        torch.cuda.synchronize()
        state.shutdown()


def test_push_gemm_reduce_scatter_norm_gather():
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
    out = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, rows in out.items():
        for i, T, err, same in rows:
            assert err < 0.05 and same, (rank, i, T, err, same)
