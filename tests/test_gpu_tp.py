"""Tensor-parallel decode (sb_open_tp) on two GPUs, one process per GPU: q|k|v,
attention and o replicated, gate/up, down and the head split by rows, the
rows exchanged over NVLink by the GEMVs themselves; MoE layers' experts spread
over the GPUs, their per-choice outputs summed by an NCCL all-reduce. Every rank's logits must
equal the single-GPU engine's bit for bit at every teacher-forced position,
and the device-resident greedy loop must pick the same ids. Skipped with
fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest

import sheep_b200
from tests import helpers

pytestmark = pytest.mark.gpu


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, path, toks, prompt, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    import sheep_b200 as sb
    res = {}
    try:
        eng = sb.Engine(path, n_ctx=128, tp=(world, rank, dist))
        try:
            res["lg"] = np.array([eng.step(int(t), p) for p, t in enumerate(toks)])
            res["ids"] = eng.generate(prompt, 16)
        finally:
            eng.close()
        if rank == 0:
            one = sb.Engine(path, n_ctx=128)
            try:
                res["lg1"] = np.array([one.step(int(t), p) for p, t in enumerate(toks)])
                res["ids1"] = one.generate(prompt, 16)
            finally:
                one.close()
    except Exception as e:   # reported, not raised: the other rank must still finish its steps
        res["error"] = repr(e)
    out[rank] = res
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("cfg,over", [
    ("tiny-q4", {}),
    ("small-q4-tied", {}),
    # a Qwen3-MoE-shaped decoder (configuration 4's features): Q/K norm, 16
    # experts top-4 spread over the GPUs, their outputs summed by NCCL
    ("tiny-q4", dict(n_expert=16, n_expert_used=4, moe_flags=1, expert_ff=256, qk_norm=1, qkv_bias=0, seed=77)),
])
def test_tensor_parallel_two_gpus_bitexact(cfg, over):
    import multiprocessing as mp
    path = helpers.model_path(sheep_b200.spec_for(cfg, **over))
    rng = np.random.default_rng(31)
    toks = rng.integers(0, 1024, 20)
    prompt = rng.integers(0, 1024, 6).astype(np.int32)
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, path, toks, prompt, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(400)
        if p.is_alive():
            p.kill()
            p.join(10)
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    r0, r1 = out[0], out[1]
    assert "error" not in r0 and "error" not in r1, (r0.get("error"), r1.get("error"))
    for r in (r0, r1):
        assert np.array_equal(r["lg"].view(np.uint32), r0["lg1"].view(np.uint32))
        assert np.array_equal(r["ids"], r0["ids1"])
