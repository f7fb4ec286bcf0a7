"""Host-side rank failure detection between lockstep steps (gloo ranks on CPU, no GPU).

A rank whose step raises records itself in the rendezvous store and leaves; its peer stops with RankFailure
naming it, at its next between-step check or when its next collective fails, well inside the collective
timeout.  A rank killed without recording anything is reported by the peer's next collective.
"""
import os
import socket
import time

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _leave(q, code):
    q.close()
    q.join_thread()  # the queued result reaches the parent before the process ends
    os._exit(code)


def _worker(rank, world, port, mode, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import torch.distributed as dist

    from vllm_suffix_hybrid_b200.parallel import state
    from vllm_suffix_hybrid_b200.parallel.health import RankFailure, RankHealth

    st = state.init(tp=world, backend="gloo", timeout_s=20)
    health = RankHealth.from_process_group()
    t0 = time.time()
    try:
        for step in range(50):
            health.check()
            box = [step if rank == 0 else None]
            try:
                dist.broadcast_object_list(box, src=0, group=st.cpu_group)
            except Exception as err:
                raise health.explain(err) from err
            if rank == 1 and step == 3:  # the injected failure, on the host, between steps
                if mode == "raise":
                    health.report("injected step failure")
                    q.put((rank, "left", None, time.time() - t0))
                    _leave(q, 0)
                q.put((rank, "killed", None, time.time() - t0))
                _leave(q, 1)  # dies without recording anything
            time.sleep(0.01)
        q.put((rank, "finished", None, time.time() - t0))
    except RankFailure as f:
        q.put((rank, "failure", (f.rank, str(f)), time.time() - t0))
    _leave(q, 0)


@pytest.mark.parametrize("mode", ["raise", "kill"])
def test_peer_failure_is_reported_not_waited_for(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, what, info, dt = q.get(timeout=120)
        res[rank] = (what, info, dt)
    for p in procs:
        p.join(timeout=60)
    assert res[1][0] == ("left" if mode == "raise" else "killed")
    what, info, dt = res[0]
    assert what == "failure", res
    if mode == "raise":
        assert info[0] == 1 and "injected step failure" in info[1]
    else:
        assert info[0] == -1 and "no rank recorded" in info[1]
    assert dt < 60  # well before any test timeout: detected, not hung


def test_single_rank_health_is_a_no_op():
    from vllm_suffix_hybrid_b200.parallel.health import RankHealth

    h = RankHealth()
    h.report("x")
    h.check()
    assert h.failed() is None
