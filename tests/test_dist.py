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


def _ep_worker(rank, world, port, out):
    """Expert parallelism's exchange on the CPU restatement: this rank computes
    the per-choice outputs of the experts it holds (zeros elsewhere), the ranks
    sum them (gloo all-reduce), and the combine in choice order must equal the
    whole layer computed in one place, bit for bit."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import numpy as np
    import torch
    import sheep_b200
    from sheep_b200 import dist as sd
    from tests import helpers
    d = sd.init("gloo", timeout_s=120)
    path = helpers.model_path(sheep_b200.spec_for("tiny-q4", n_layer=1, n_expert=16, n_expert_used=4, moe_flags=1,
                                                  expert_ff=256, seed=901))
    orc = helpers.Oracle(path, 16)
    x = np.random.default_rng(5).standard_normal((6, orc.info[1])).astype(np.float32)
    y_full, sel, w = orc.moe_ffn(0, x)
    lo, hi = sd.expert_range(16, world, rank)
    yk = np.zeros((len(x), sel.shape[1], orc.info[1]), np.float32)
    for t in range(len(x)):
        for j in range(sel.shape[1]):
            if lo <= sel[t, j] < hi:
                yk[t, j] = orc.moe_expert(0, int(sel[t, j]), x[t])
    tk = torch.from_numpy(yk)
    d.all_reduce(tk)
    yk = tk.numpy()
    # the combine in choice order, as the layer computes it (fused multiply-adds)
    y = np.zeros_like(y_full)
    wk = np.ascontiguousarray(w, np.float32)
    yk = np.ascontiguousarray(yk, np.float32)
    orc.lib().so_moe_combine(len(x), sel.shape[1], orc.info[1], helpers._p(wk), helpers._p(yk), helpers._p(y))
    out[rank] = (bool(np.array_equal(y.view(np.uint32), y_full.view(np.uint32))), (lo, hi))
    orc.close()
    d.barrier()
    d.destroy_process_group()


def test_expert_parallel_exchange_two_gloo_ranks():
    import multiprocessing as mp
    from tests import helpers
    helpers.build_oracle()
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    ps = [ctx.Process(target=_ep_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(300)
        assert p.exitcode == 0
    assert out[0][0] and out[1][0]
    assert out[0][1] == (0, 8) and out[1][1] == (8, 16)
