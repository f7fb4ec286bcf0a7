"""Expert-parallel token exchange: device all-to-all over NVLink peer memory vs NCCL.

Run with one process per GPU (N >= 2):
  torchrun --nproc-per-node N --master-addr 127.0.0.1 -m vllm_suffix_hybrid_b200.bench.ep_bench
DeepSeek-V3.2 MoE shape (hidden 7168, 256 routed experts, top-8, data-parallel attention: every rank
routes its own T tokens).  Per T, each path is captured in a CUDA graph of `iters` calls and timed with
CUDA events; the per-call time is the max over ranks.  Exchange only (the expert GEMMs are the same on
both paths and are replaced by a copy of the received rows):
  a2a  : ep_dispatch (rows only to the ranks hosting one of the token's experts, route rows to all)
         + ep_combine (expert outputs back to the owner, summed in rank order);
  a2a_fp4: the same with the rows quantised to NVFP4 inside the dispatch (the W4A4 expert path);
  nccl : all-gather of x, ids, weights + reduce-scatter of the [N*T, H] partials (the path with
         SH_EP_A2A=0).
Roofline of the a2a: the bytes this rank sends over NVLink (rows to remote expert ranks in the
dispatch, returned rows in the combine, as measured from the routes) / 770 GB/s (measured peer-copy
bandwidth per direction); `frac` = that time / measured time.
"""
import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--hidden", type=int, default=7168)
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--tokens", default="8,32,128,512")
    ap.add_argument("--iters", type=int, default=50)
    a = ap.parse_args()
    from vllm_suffix_hybrid_b200.parallel import ep, ep_a2a, state

    W = int(os.environ.get("WORLD_SIZE", "1"))
    st = state.init(ep=W, dp=W, timeout_s=120)
    rank = st.rank
    H, E, k = a.hidden, a.experts, a.topk
    e_local = E // W
    toks = [int(t) for t in a.tokens.split(",")]
    comm = ep_a2a.get(H, ep.A2A_MAX_TOKENS, k, e_local)
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    rows = []
    for T in toks:
        x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
        ids = torch.stack([torch.randperm(E, device=dev, generator=g)[:k] for _ in range(T)]).to(torch.int32)
        w = torch.rand(T, k, device=dev, generator=g)

        def a2a():
            xs, ids_l, w_l = comm.dispatch(x, ids, w)
            return comm.combine(xs, ids)  # the received rows stand in for the expert outputs

        comm_q = ep_a2a.get(H, ep.A2A_MAX_TOKENS, k, e_local, True) if H % 256 == 0 else None

        def a2a_fp4():  # NVFP4 rows (the W4A4 expert path); bf16 expert outputs come back
            comm_q.dispatch(x, ids, w)
            return comm_q.combine(comm_q.x_buf[: W * T * H].view(W * T, H), ids)

        def nccl():
            xs = ep._all_gather(x)
            ids_a = ep._all_gather(ids)
            w_a = ep._all_gather(w)
            return ep._reduce_scatter(xs)

        res = {}
        paths = [("a2a", a2a), ("nccl", nccl)] + ([("a2a_fp4", a2a_fp4)] if comm_q is not None else [])
        for name, fn in paths:
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            dist.barrier()
            graph = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                with torch.cuda.graph(graph):
                    for _ in range(a.iters):
                        fn()
            torch.cuda.synchronize()
            dist.barrier()
            graph.replay()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            e1.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) * 1000.0 / a.iters], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            res[name] = t.item()
            del graph
        comm.check()
        if comm_q is not None:
            comm_q.check()
        # bytes this rank sends over NVLink in the a2a (dispatch rows to remote expert ranks + returned rows)
        dests = torch.zeros(T, W, dtype=torch.bool, device=dev)
        dests.scatter_(1, (ids.long() // e_local), True)
        remote_out = int(dests.sum().item()) - int(dests[:, rank].sum().item())
        sent = torch.tensor([remote_out * H * 2.0], device=dev)
        dist.all_reduce(sent, op=dist.ReduceOp.MAX)
        link_us = 2 * sent.item() / (LINK_GBS * 1e3)  # dispatch + combine, per direction
        rows.append({"T_per_rank": T, "a2a_us": round(res["a2a"], 2), "nccl_us": round(res["nccl"], 2),
                     "a2a_fp4_dispatch_us": round(res.get("a2a_fp4", 0.0), 2),
                     "speedup": round(res["nccl"] / res["a2a"], 2), "link_bound_us": round(link_us, 2),
                     "frac_of_link_roofline": round(link_us / res["a2a"], 3)})
    if rank == 0:
        for r in rows:
            print(json.dumps({"world": W, "hidden": H, "experts": E, "topk": k, **r}))
    torch.cuda.synchronize()
    state.shutdown()


if __name__ == "__main__":
    main()
