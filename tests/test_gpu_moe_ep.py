"""Expert-parallel MoE layer (sb_moe_open_ep) on two GPUs: one process per GPU,
the experts split between them, every process passing all tokens. Each rank's
output must equal the single-GPU layer's bit for bit (the per-choice outputs
are summed with exact zeros and combined in choice order). Skipped with fewer
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


def _run(ctx, jobs, timeout=300):
    ps = [ctx.Process(target=_worker, args=a) for a in jobs]
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
