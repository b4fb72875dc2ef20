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


def test_a2a_plan_invariants():
    """The all-to-all exchange's host plan (sb_moe_a2a_plan, this library's own
    code; no GPU): every (token, choice) row of a rank goes to the one rank
    holding its expert, grouped by destination in slot order; what rank r sends
    to rank d is exactly what d expects from r, in the same order; received
    rows carry their experts, all held by the receiver; the dispatch cuts each
    expert's rows into chunks of at most 8."""
    import numpy as np
    import sheep_b200
    from sheep_b200 import dist as sd
    rng = np.random.default_rng(3)
    for world in (2, 3, 4, 8):
        for ne, k in ((16, 4), (128, 8), (24, 2)):
            if ne < world:
                continue
            sels = []
            for _ in range(world):
                n = int(rng.integers(0, 9))
                sels.append(np.array([rng.choice(ne, k, replace=False) for _ in range(n)], np.int64).reshape(n, k))
            owner = lambda e: next(r for r in range(world) if sd.expert_range(ne, world, r)[0] <= e < sd.expert_range(ne, world, r)[1])
            plans = [sheep_b200.moe_a2a_plan(world, r, ne, sels) for r in range(world)]
            for r, (scnt, rcnt, sslot, rexp, nch) in enumerate(plans):
                T = len(sels[r])
                assert scnt.sum() == T * k
                want = [t * k + j for d in range(world) for t in range(T) for j in range(k) if owner(sels[r][t, j]) == d]
                assert sslot.tolist() == want
                lo, hi = sd.expert_range(ne, world, r)
                assert all(lo <= e < hi for e in rexp)
                exp_rows = [int(sels[s_][t, j]) for s_ in range(world) for t in range(len(sels[s_])) for j in range(k)
                            if owner(sels[s_][t, j]) == r]
                assert rexp.tolist() == exp_rows
                for s_ in range(world):
                    assert rcnt[s_] == plans[s_][0][r]
                counts = np.bincount(rexp, minlength=ne) if len(rexp) else np.zeros(ne, int)
                assert nch == int(sum((c + 7) // 8 for c in counts))


def _a2a_worker(rank, world, port, out):
    """Expert parallelism by all-to-all on the CPU restatement: each rank holds
    its own tokens and the experts of its range; the choices are exchanged,
    each (token, choice) row is sent to the rank holding its expert (as the
    library's plan says), that rank runs the expert, the result comes back to
    its slot and the combine runs in choice order -- equal to the whole layer
    over this rank's tokens computed in one place, bit for bit."""
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
    E = orc.info[1]
    x = np.random.default_rng(50 + rank).standard_normal((3 + 4 * rank, E)).astype(np.float32)
    y_full, sel, w = orc.moe_ffn(0, x)
    k = sel.shape[1]
    sels = [None] * world
    d.all_gather_object(sels, np.asarray(sel))
    scnt, rcnt, sslot, rexp, _ = sheep_b200.moe_a2a_plan(world, rank, 16, sels)
    soff, roff = np.concatenate([[0], np.cumsum(scnt)]), np.concatenate([[0], np.cumsum(rcnt)])

    def exchange(rows_out, cnt_out, off_out, cnt_in, off_in):
        rows_in = np.zeros((int(cnt_in.sum()), E), np.float32)
        rows_in[off_in[rank]:off_in[rank] + cnt_in[rank]] = rows_out[off_out[rank]:off_out[rank] + cnt_out[rank]]
        reqs, bufs = [], {}
        for p in range(world):
            if p == rank:
                continue
            if cnt_out[p]:
                reqs.append(d.isend(torch.from_numpy(np.ascontiguousarray(rows_out[off_out[p]:off_out[p] + cnt_out[p]])), p))
            if cnt_in[p]:
                bufs[p] = torch.zeros((int(cnt_in[p]), E), dtype=torch.float32)
                reqs.append(d.irecv(bufs[p], p))
        for q in reqs:
            q.wait()
        for p, b in bufs.items():
            rows_in[off_in[p]:off_in[p] + cnt_in[p]] = b.numpy()
        return rows_in

    recv = exchange(x[sslot // k], scnt, soff, rcnt, roff)                   # dispatch
    res = np.stack([orc.moe_expert(0, int(e), r) for e, r in zip(rexp, recv)]) if len(rexp) else recv
    back = exchange(res, rcnt, roff, scnt, soff)                              # combine
    yk = np.zeros((len(x) * k, E), np.float32)
    yk[sslot] = back
    y = np.zeros_like(y_full)
    wk = np.ascontiguousarray(w, np.float32)
    orc.lib().so_moe_combine(len(x), k, E, helpers._p(wk), helpers._p(yk), helpers._p(y))
    out[rank] = bool(np.array_equal(y.view(np.uint32), y_full.view(np.uint32)))
    orc.close()
    d.barrier()
    d.destroy_process_group()


def test_expert_parallel_all_to_all_two_gloo_ranks():
    import multiprocessing as mp
    from tests import helpers
    helpers.build_oracle()
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    ps = [ctx.Process(target=_a2a_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(300)
        assert p.exitcode == 0
    assert out[0] and out[1]
