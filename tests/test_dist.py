"""The bench's multi-rank plumbing on CPU: two gloo ranks, max over ranks and
the weak-scaling aggregate (no GPU)."""
import os
import socket

import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    from sheep_b200 import dist as sd
    d = sd.init("gloo", timeout_s=60)
    # rank r "took" 1.0 + r seconds for 10 tokens
    m = sd.max_over_ranks(d, 1.0 + rank, device="cpu")
    out[rank] = (m, sd.replica_throughput(10, m, world))
    d.barrier()
    d.destroy_process_group()


def test_two_gloo_ranks():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(120)
        assert p.exitcode == 0
    assert out[0] == out[1] == (2.0, 10.0)


def test_single_rank_needs_no_group():
    from sheep_b200 import dist as sd
    assert sd.max_over_ranks(None, 3.5) == 3.5
    assert sd.replica_throughput(100, 2.0, 1) == pytest.approx(50.0)
