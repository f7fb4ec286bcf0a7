"""Expert-parallel all-to-all (dispatch / experts / combine over NVLink peer memory) on 2+ GPUs.

Every rank routes its own tokens over all experts; the device all-to-all path must match the fp32
sum over the routed experts computed from all ranks' weights, agree with the NCCL all-gather /
reduce-scatter path, survive consecutive calls of different sizes (single receive buffers ordered by
the epoch barriers) and replay correctly from a CUDA graph.  The NVFP4-quantising dispatch and the
dispatch that runs the router top-k itself must be bit-identical to the unfused paths.  Skipped with
fewer than two GPUs.
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


class _Moe:
    def __init__(self, w13, w2, e_local, F):
        self.w13, self.w2, self.E_local, self.F = w13, w2, e_local, F
        self.fp4 = None
        self.fp8 = None


def _reference(x_all, ids_all, w_all, w13_all, w2_all, F):
    """fp32 sum over routed experts with the same bf16 rounding points as the grouped expert path."""
    T, H = x_all.shape
    out = torch.zeros(T, H)
    for t in range(T):
        for j in range(ids_all.shape[1]):
            e = int(ids_all[t, j])
            gu = x_all[t].float() @ w13_all[e * 2 * F:(e + 1) * 2 * F].float().t()
            a = (torch.nn.functional.silu(gu[:F]) * gu[F:]).to(torch.bfloat16).float()
            out[t] += (a @ w2_all[e * H:(e + 1) * H].float().t()).to(torch.bfloat16).float() * float(w_all[t, j])
    return out


def _worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from vllm_suffix_hybrid_b200.parallel import ep, state

    state.init(ep=world, dp=world, backend="nccl", timeout_s=60)
    try:
        H, F, E, k = 512, 128, 4 * world, 3
        e_local = E // world
        g = torch.Generator().manual_seed(11)
        w13_all = (torch.randn(E * 2 * F, H, generator=g) * 0.05).to(torch.bfloat16)
        w2_all = (torch.randn(E * H, F, generator=g) * 0.05).to(torch.bfloat16)
        e0 = rank * e_local
        moe = _Moe(w13_all[e0 * 2 * F:(e0 + e_local) * 2 * F].cuda(), w2_all[e0 * H:(e0 + e_local) * H].cuda(),
                   e_local, F)
        results = {}
        for call, T in enumerate([37, 5, 64, 1, 37]):
            gi = torch.Generator().manual_seed(1000 * call + rank)
            x = (torch.randn(T, H, generator=gi)).to(torch.bfloat16)
            ids = torch.stack([torch.randperm(E, generator=gi)[:k] for _ in range(T)]).to(torch.int32)
            w = torch.rand(T, k, generator=gi)
            os.environ["SH_EP_A2A"] = "1"
            got = ep.dp_dispatch_combine(moe, x.cuda(), ids.cuda(), w.cuda())
            os.environ["SH_EP_A2A"] = "0"
            nccl = ep.dp_dispatch_combine(moe, x.cuda(), ids.cuda(), w.cuda())
            torch.cuda.synchronize()
            ref = _reference(x, ids, w, w13_all, w2_all, F)
            scale = ref.abs().max().item()
            results[f"{call}:T{T}"] = ((got.float().cpu() - ref).abs().max().item() / scale,
                                       (got.float() - nccl.float()).abs().max().item() / scale)
        # CUDA-graph replay: same pointers every call, the epochs advance on the device.
        os.environ["SH_EP_A2A"] = "1"
        T = 16
        xg = torch.zeros(T, H, dtype=torch.bfloat16, device="cuda")
        idg = torch.zeros(T, k, dtype=torch.int32, device="cuda")
        wg = torch.zeros(T, k, device="cuda")
        ep.dp_dispatch_combine(moe, xg, idg, wg)  # warm-up (creates the communicator for T <= max)
        torch.cuda.synchronize()
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph):
                og = ep.dp_dispatch_combine(moe, xg, idg, wg)
        torch.cuda.synchronize()
        for rep in range(3):
            gi = torch.Generator().manual_seed(50 + 7 * rep + rank)
            x = torch.randn(T, H, generator=gi).to(torch.bfloat16)
            ids = torch.stack([torch.randperm(E, generator=gi)[:k] for _ in range(T)]).to(torch.int32)
            w = torch.rand(T, k, generator=gi)
            xg.copy_(x)
            idg.copy_(ids)
            wg.copy_(w)
            torch.cuda.synchronize()
            dist.barrier()
            graph.replay()
            torch.cuda.synchronize()
            ref = _reference(x, ids, w, w13_all, w2_all, F)
            results[f"graph{rep}"] = ((og.float().cpu() - ref).abs().max().item() / ref.abs().max().item(), 0.0)
        del graph
        # NVFP4 (W4A4) experts: the quantising dispatch must reproduce the bf16 dispatch bit for bit (the rows
        # are quantised once by the dispatch instead of by the receiver, with the same math).
        from vllm_suffix_hybrid_b200.ops import reference as ref

        def quant(wt, rows):
            ps, ss, gs = [], [], []
            for e in range(e_local):
                gsc = ref.nvfp4_global_scale(wt[e * rows:(e + 1) * rows])
                pk, sc = ref.nvfp4_quantize(wt[e * rows:(e + 1) * rows], gsc)
                ps.append(pk), ss.append(sc), gs.append(gsc.reshape(1).float())
            return tuple(t.cuda() for t in (torch.cat(ps), torch.cat(ss), torch.cat(gs)))

        H4 = 256
        w13_4 = (torch.randn(E * 2 * F, H4, generator=g) * 0.05).to(torch.bfloat16)
        w2_4 = (torch.randn(E * H4, F, generator=g) * 0.05).to(torch.bfloat16)
        moe4 = _Moe(None, None, e_local, F)
        moe4.fp4 = (quant(w13_4[e0 * 2 * F:(e0 + e_local) * 2 * F], 2 * F), quant(w2_4[e0 * H4:(e0 + e_local) * H4], H4))
        for call, T in enumerate([21, 3, 40]):
            gi = torch.Generator().manual_seed(300 + 10 * call + rank)
            x = torch.randn(T, H4, generator=gi).to(torch.bfloat16).cuda()
            ids = torch.stack([torch.randperm(E, generator=gi)[:k] for _ in range(T)]).to(torch.int32).cuda()
            w = torch.rand(T, k, generator=gi).cuda()
            os.environ["SH_EP_A2A_FP4"] = "1"
            got = ep.dp_dispatch_combine(moe4, x, ids, w)
            os.environ["SH_EP_A2A_FP4"] = "0"
            base = ep.dp_dispatch_combine(moe4, x, ids, w)
            torch.cuda.synchronize()
            results[f"fp4:{call}:T{T}"] = (0.0 if torch.equal(got, base) else 1.0, 0.0)
        os.environ["SH_EP_A2A_FP4"] = "1"
        # Router top-k inside the dispatch kernel: bit-identical to ops.moe_route + the same dispatch, for the
        # softmax and the sigmoid group-limited routers, with bf16 and NVFP4 experts.
        from vllm_suffix_hybrid_b200 import ops

        bias = (torch.randn(E, generator=g) * 0.1).cuda()
        routers = (dict(sigmoid_grouped=False, bias=None, n_groups=1, topk_groups=1, renorm=True, scale=1.0),
                   dict(sigmoid_grouped=True, bias=bias, n_groups=2, topk_groups=1, renorm=True, scale=2.5))
        for mi, (mdl, HH) in enumerate(((moe, H), (moe4, H4))):
            mdl.k = k
            for ri, args in enumerate(routers):
                mdl.route_args = lambda a=args: a
                for call, T in enumerate([19, 2]):
                    gi = torch.Generator().manual_seed(700 + 10 * call + rank)
                    x = torch.randn(T, HH, generator=gi).to(torch.bfloat16).cuda()
                    logits = torch.randn(T, E, generator=gi).to(torch.bfloat16).cuda()
                    got = ep.dp_route_dispatch_combine(mdl, x, logits)
                    ids, w = ops.moe_route(logits, k, **args)
                    base = ep.dp_dispatch_combine(mdl, x, ids, w)
                    torch.cuda.synchronize()
                    results[f"route:{mi}:{ri}:{call}"] = (0.0 if torch.equal(got, base) else 1.0, 0.0)
        # The experts' weighted sum stored straight into the owners' return rows (default) must equal the
        # local combine + copy (SH_EP_COMBINE_PUSH=0) bit for bit.
        for mi, (mdl, HH) in enumerate(((moe, H), (moe4, H4))):
            mdl.route_args = lambda a=routers[1]: a
            for call, T in enumerate([23, 1]):
                gi = torch.Generator().manual_seed(900 + 10 * call + rank)
                x = torch.randn(T, HH, generator=gi).to(torch.bfloat16).cuda()
                logits = torch.randn(T, E, generator=gi).to(torch.bfloat16).cuda()
                os.environ["SH_EP_COMBINE_PUSH"] = "0"
                base = ep.dp_route_dispatch_combine(mdl, x, logits)
                os.environ["SH_EP_COMBINE_PUSH"] = "1"
                got = ep.dp_route_dispatch_combine(mdl, x, logits)
                torch.cuda.synchronize()
                results[f"push:{mi}:{call}"] = (0.0 if torch.equal(got, base) else 1.0, 0.0)
        from vllm_suffix_hybrid_b200.parallel import ep_a2a

        assert any(c.quant for c in ep_a2a._comms.values())
        for c in ep_a2a._comms.values():
            c.check()
        q.put((rank, results))
    finally:
        torch.cuda.synchronize()
        state.shutdown()


def test_ep_all_to_all_multi_gpu():
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
    for rank, calls in res.items():
        for name, (e_ref, e_nccl) in calls.items():
            assert e_ref < 0.02 and e_nccl < 0.02, (rank, name, e_ref, e_nccl)
