"""sml-gpu-fwd on the GPU, read with the reference's own parsers of its
output (tooling/sml_tune.py:98-99 RE_GPU / RE_GPU_GRADE, and the agreement
rule of mlmi/backend/orchestrator.py parse_gpu_agreement: corr >= 0.999).

The grade compares the GPU's logits, position by position over the given ids,
with the CPU engine's saved in the reference sml-cli's SML_ALL_LOGITS layout
(here written from the reference build, oracle/_ref): this engine computes the
reference's arithmetic, so the correlation is 1 and every top token agrees.
"""
import os
import re
import subprocess

import numpy as np
import pytest

import sheep_b200
from sheep_b200 import build
from tests import helpers

pytestmark = pytest.mark.gpu

RE_GPU = re.compile(r"= ([0-9.]+) tok/s")
RE_GPU_GRADE = re.compile(r"mean logit corr ([0-9.]+), worst ([0-9.]+), top-1 agree (\d+)/(\d+)")


def _run(args, env=None, timeout=300):
    e = dict(os.environ)
    e.update(env or {})
    r = subprocess.run([build.build_cli()] + args, capture_output=True, text=True, timeout=timeout, env=e)
    return r.returncode, r.stdout


@pytest.mark.skipif(not helpers.have_ref(), reason="reference CPU build (oracle/_ref) not present")
def test_cli_grade_and_speed_lines(tmp_path):
    path = helpers.model_path(sheep_b200.spec_for("small-q4-tied"))
    ids = [int(t) for t in np.random.default_rng(17).integers(0, 4096, 12)]
    lg = helpers.ref("forward", path, tokens=ids, n_ctx=128)
    f = tmp_path / "cpu.logits"
    with open(f, "wb") as fh:
        np.array([lg.shape[1], len(ids)], np.int32).tofile(fh)
        np.ascontiguousarray(lg, np.float32).tofile(fh)
    rc, out = _run([path, ",".join(map(str, ids)), "16"], {"SML_CPU_LOGITS": str(f), "SML_CTX": "128"})
    print(out)
    assert rc == 0, out
    m = RE_GPU_GRADE.search(out)
    assert m, out
    corr, worst, agree, of = float(m.group(1)), float(m.group(2)), int(m.group(3)), int(m.group(4))
    assert (corr, worst, agree, of) == (1.0, 1.0, len(ids), len(ids))
    speeds = [float(v) for v in RE_GPU.findall(out)]
    assert len(speeds) == 1 and speeds[0] > 0        # the graph-replay line ("= X tok/s")
    assert "per-token path" in out and "tokens identical to the per-token path" in out


def test_cli_logits_out_and_prompt_timing(tmp_path):
    path = helpers.model_path(sheep_b200.spec_for("tiny-q4"))
    ids = [int(t) for t in np.random.default_rng(18).integers(0, 1024, 40)]
    f = tmp_path / "next.logits"
    rc, out = _run([path, ",".join(map(str, ids)), "0"], {"SML_LOGITS_OUT": str(f), "SML_CTX": "128"})
    assert rc == 0, out
    raw = np.fromfile(f, np.int32, 2)
    got = np.fromfile(f, np.float32, offset=8)
    assert raw[0] == 1024 and raw[1] == 0 and got.size == 1024
    eng = sheep_b200.Engine(path, n_ctx=128)
    try:
        eng.prompt_mode(2)
        want = eng.prefill(np.array(ids, np.int32))
    finally:
        eng.close()
    assert np.array_equal(got.view(np.uint32), np.asarray(want, np.float32).view(np.uint32))
    rc, out = _run([path, ",".join(map(str, ids)), "0"], {"SML_PP": "16,64,999", "SML_CTX": "128"})
    assert rc == 0, out
    assert re.search(r"GPU prompt +16 tokens: [0-9.]+ ms = [0-9.]+ tok/s", out), out
    assert re.search(r"GPU prompt +64 tokens: [0-9.]+ ms = [0-9.]+ tok/s", out), out
    assert "prompt 999 skipped" in out


def test_cli_without_cpu_logits_says_no_comparison_ran():
    path = helpers.model_path(sheep_b200.spec_for("tiny-q4"))
    rc, out = _run([path, "1,2,3", "8"], {"SML_CTX": "128"})
    assert rc == 0, out
    assert "no comparison ran" in out and not RE_GPU_GRADE.search(out)
    rc, out = _run(["/nonexistent.ssf", "1,2,3", "8"])
    assert rc == 1
