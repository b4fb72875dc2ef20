"""Expert-parallel MoE layer (sb_moe_open_ep) on two GPUs: one process per GPU,
the experts split between them. With the all-reduce exchange every process
passes all tokens; with the all-to-all exchange (sb_moe_set_exchange) each
passes its own. Either way each rank's output must equal the single-GPU
layer's rows bit for bit (the per-choice outputs are summed with exact zeros,
or sent back to their slots, and combined in choice order). Skipped with fewer
than two GPUs."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _worker(gpu, world, rank, nid, path, xs, out):
    os.environ["CUDA_VISIBLE_DEVICES"] = str(gpu)
    os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import sheep_b200
    m = sheep_b200.MoeLayer(path, 0, max_tokens=64, ep=None if world == 1 else (world, rank, nid))
    res = []
    for x in xs:
        y, sel, w, na = m.forward(x)
        res.append((y, sel, w, na))
    out[(world, rank)] = (res, (m.e_lo, m.e_hi))
    m.close()


def _run(ctx, jobs, timeout=300, target=None):
    ps = [ctx.Process(target=target or _worker, args=a) for a in jobs]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout)
    for p in ps:
        if p.is_alive():   # a rank stuck in NCCL setup: end this test's own children
            p.kill()
            p.join(10)
    return [p.exitcode for p in ps]


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_moe_expert_parallel_two_gpus_bitexact():
    import multiprocessing as mp
    import sheep_b200
    from tests import helpers
    os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
    path = helpers.model_path(sheep_b200.spec_for("tiny-q4", n_layer=1, n_embd=512, n_expert=16, n_expert_used=4,
                                                  moe_flags=1, expert_ff=256, seed=902))
    rng = np.random.default_rng(12)
    xs = [rng.standard_normal((t, 512)).astype(np.float32) for t in (1, 16, 64)]
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    assert _run(ctx, [(0, 1, 0, b"", path, xs, out)]) == [0]
    nid = sheep_b200.nccl_unique_id()   # this process hosts the id's bootstrap root
    assert _run(ctx, [(r, 2, r, nid, path, xs, out) for r in range(2)]) == [0, 0]
    ref, _ = out[(1, 0)]
    assert out[(2, 0)][1] == (0, 8) and out[(2, 1)][1] == (8, 16)
    for r in range(2):
        res, _ = out[(2, r)]
        for (y, sel, w, na), (yr, selr, wr, nar) in zip(res, ref):
            assert np.array_equal(sel, selr) and np.array_equal(w.view(np.uint32), wr.view(np.uint32))
            assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))
            assert na <= nar   # this rank reads only the chosen experts it holds


def _int_worker(gpu, world, rank, nid, path, xs, out):
    """The single-GPU layer on the integer kernels (the expert products the
    all-to-all exchange runs)."""
    os.environ["CUDA_VISIBLE_DEVICES"] = str(gpu)
    import sheep_b200
    m = sheep_b200.MoeLayer(path, 0, max_tokens=256)
    m.tensor_cores(False)
    out[(world, rank)] = ([m.forward(x) for x in xs], None)
    m.close()


def _a2a_worker(gpu, world, rank, nid, path, xs, out):
    """Rank `rank` passes its own rows xs[case][rank] through the all-to-all exchange."""
    os.environ["CUDA_VISIBLE_DEVICES"] = str(gpu)
    os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import sheep_b200
    m = sheep_b200.MoeLayer(path, 0, max_tokens=64, ep=(world, rank, nid))
    m.exchange("all-to-all")
    out[(world, rank)] = [m.forward(rows[rank]) for rows in xs]
    m.close()


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_moe_expert_parallel_all_to_all_two_gpus_bitexact():
    """Each GPU passes its own tokens (ragged counts, one token each too): the
    choices are exchanged, the rows travel to the GPU holding their expert and
    back; every rank's outputs, choices and weights equal the single-GPU
    layer's rows for its tokens, bit for bit."""
    import multiprocessing as mp
    import sheep_b200
    from tests import helpers
    os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
    path = helpers.model_path(sheep_b200.spec_for("tiny-q4", n_layer=1, n_embd=512, n_expert=16, n_expert_used=4,
                                                  moe_flags=1, expert_ff=256, seed=902))
    rng = np.random.default_rng(13)
    counts = [(1, 1), (16, 5), (64, 64), (3, 40)]
    xs = [[rng.standard_normal((t, 512)).astype(np.float32) for t in c] for c in counts]
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    # the single-GPU layer over both ranks' rows at once
    whole = [np.concatenate(rows) for rows in xs]
    assert _run(ctx, [(0, 1, 0, b"", path, whole, out)], target=_int_worker) == [0]
    ref, _ = out[(1, 0)]
    nid = sheep_b200.nccl_unique_id()
    assert _run(ctx, [(r, 2, r, nid, path, xs, out) for r in range(2)], target=_a2a_worker) == [0, 0]
    for c, (t0, t1) in enumerate(counts):
        yr, selr, wr, _ = ref[c]
        for r, (a, b) in enumerate(((0, t0), (t0, t0 + t1))):
            y, sel, w, na = out[(2, r)][c]
            assert np.array_equal(sel, selr[a:b]) and np.array_equal(w.view(np.uint32), wr[a:b].view(np.uint32))
            assert np.array_equal(y.view(np.uint32), yr[a:b].view(np.uint32)), (c, r)
