"""Whole-decode parity on the GPU, bit for bit.

The engine computes every float operation of the reference's CPU decode in the
reference's order (the matvec accumulator chains and their fused
multiply-adds, RMSNorm, RoPE, the attention's chains and sequential softmax sum
with the host libm's expf, the SiLU's own exponential, the residual adds), so
its logits equal the reference build's -- and the oracle's, which is pinned to
it bit for bit -- exactly. The tests compare logits as bit patterns and greedy
ids with strict equality; teacher-forced runs feed both engines the same
tokens, free-running runs let each choose its own.
"""
import numpy as np
import pytest

import sheep_b200
from tests import helpers

pytestmark = pytest.mark.gpu

WIDTHS = [(nb, six) for six in (0, 1) for nb in (2, 3, 4, 5, 6, 7, 8)]


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _first_diff(a, b):
    """(step, count) of the first step whose logits differ, or None."""
    for k in range(len(a)):
        n = int((_bits(a[k]) != _bits(b[k])).sum())
        if n:
            return k, n
    return None


def _teacher_forced(path, tokens, n_ctx=128):
    eng = sheep_b200.Engine(path, n_ctx=n_ctx)
    orc = helpers.Oracle(path, n_ctx=n_ctx)
    try:
        got = np.array([eng.step(int(t), pos) for pos, t in enumerate(tokens)])
        want = np.array([orc.forward(int(t), pos) for pos, t in enumerate(tokens)])
    finally:
        eng.close()
        orc.close()
    return got, want


@pytest.mark.parametrize("cfg", ["tiny-q4", "small-q4-tied"])
def test_decode_bit_exact_against_oracle(cfg):
    """40 teacher-forced positions (past one 64-position V stage of the
    attention): every logit bit-equal to the oracle's."""
    path = helpers.model_path(sheep_b200.spec_for(cfg))
    toks = np.random.default_rng(3).integers(0, 1024, 70)
    got, want = _teacher_forced(path, toks)
    assert _first_diff(got, want) is None, _first_diff(got, want)


def test_decode_long_context_bit_exact():
    """Positions past the attention's 192 staged rows (keys read in place,
    values through double-buffered blocks of 96 rows): 300 teacher-forced
    positions, two blocks and a partial one past the staged rows, every logit
    bit-equal to the oracle's."""
    path = helpers.model_path(sheep_b200.spec_for("tiny-q4"))
    toks = np.random.default_rng(31).integers(0, 1024, 300)
    got, want = _teacher_forced(path, toks, n_ctx=320)
    assert _first_diff(got, want) is None, _first_diff(got, want)


@pytest.mark.parametrize("nb,six", WIDTHS)
def test_decode_every_width_bit_exact(nb, six):
    """Every code width Q2..Q8 with 8- and 6-bit group fields: the ladder,
    flat and bit-plane epilogues, and their sums, as the reference's dispatch
    runs them."""
    spec = sheep_b200.spec_for("tiny-q4", nbits=nb, emb_nbits=nb, scale6=six, minneg=six, seed=9)
    path = helpers.model_path(spec)
    toks = np.random.default_rng(4).integers(0, 1024, 12)
    got, want = _teacher_forced(path, toks, n_ctx=64)
    assert _first_diff(got, want) is None, _first_diff(got, want)


def test_greedy_ids_first_32_steps():
    """Free-running greedy decode: 32 generated ids equal the oracle's."""
    path = helpers.model_path(sheep_b200.spec_for("tiny-q4"))
    prompt = np.random.default_rng(11).integers(0, 1024, 8).astype(np.int32)
    eng = sheep_b200.Engine(path, n_ctx=128)
    orc = helpers.Oracle(path, n_ctx=128)
    try:
        got = eng.generate(prompt, 32)
        want, _ = orc.decode(prompt, 32)
    finally:
        eng.close()
        orc.close()
    assert np.array_equal(got, want), (got, want)


def test_generate_equals_stepping():
    """The device-resident greedy loop chooses what stepping + host argmax chooses."""
    path = helpers.model_path(sheep_b200.spec_for("small-q4-tied"))
    prompt = np.array([5, 17, 400, 3, 99], np.int32)
    eng = sheep_b200.Engine(path, n_ctx=128)
    try:
        got = eng.generate(prompt, 20)
        lg = None
        for i, t in enumerate(prompt):
            lg = eng.step(int(t), i)
        ids = []
        pos = len(prompt)
        for _ in range(20):
            t = int(np.argmax(lg))
            ids.append(t)
            lg = eng.step(t, pos)
            pos += 1
        assert np.array_equal(got, np.array(ids, np.int32))
        # and the run is deterministic
        assert np.array_equal(eng.generate(prompt, 20), got)
    finally:
        eng.close()


def test_reference_api_errors():
    """sml-gpu.h error behaviour: 0 + reason on open failure, NULL past n_ctx."""
    ok, why = sheep_b200.sml_gpu_open("/nonexistent/model.ssf", 64)
    assert ok == 0 and why
    path = helpers.model_path(sheep_b200.spec_for("tiny-q4"))
    ok, why = sheep_b200.sml_gpu_open(path, 64)
    assert ok == 1, why
    try:
        assert sheep_b200.sml_gpu_step(1, 64) is None            # pos >= n_ctx
        assert sheep_b200.sml_gpu_prefill([1, 2, 3], 62) is None  # pos0 + n > n_ctx
        lg = sheep_b200.sml_gpu_step(1, 0)
        assert lg is not None and lg.shape == (1024,) and np.isfinite(lg).all()
        assert sheep_b200.sml_gpu_layers() == (2, 2)
        assert sheep_b200.sml_gpu_decode_cpu(1) == 0
        lp = sheep_b200.sml_gpu_prefill([1, 2, 3], 0)
        lq = sheep_b200.sml_gpu_prefill([1, 2, 3], 0)
        assert np.array_equal(lp, lq)
    finally:
        sheep_b200.sml_gpu_close()


@pytest.mark.skipif(not helpers.have_ref(), reason="reference CPU build (oracle/_ref) not present")
def test_decode_bit_exact_against_reference_build():
    """The reference's own CPU decode (oracle/_ref, its unchanged sources),
    teacher-forced: logits bit-equal at every position."""
    path = helpers.model_path(sheep_b200.spec_for("small-q4-tied"))
    toks = np.random.default_rng(8).integers(0, 4096, 24)
    ref_lg = helpers.ref("forward", path, tokens=[int(t) for t in toks], n_ctx=128)
    eng = sheep_b200.Engine(path, n_ctx=128)
    try:
        got = np.array([eng.step(int(t), pos) for pos, t in enumerate(toks)])
    finally:
        eng.close()
    assert _first_diff(got, ref_lg) is None, _first_diff(got, ref_lg)


def _cfg0_run(eng, prompt, ngen):
    """Stepped greedy decode through the engine: ids and the logits that chose them."""
    lg = None
    for i, t in enumerate(prompt):
        lg = eng.step(int(t), i)
    ids, lgs = [], []
    for g in range(ngen):
        t = int(np.argmax(lg))      # the first largest, as sml_sample_greedy takes it
        ids.append(t)
        lgs.append(lg)
        if g + 1 < ngen:
            lg = eng.step(t, len(prompt) + g)
    return np.array(ids, np.int32), np.array(lgs)


@pytest.mark.skipif(not helpers.have_ref(), reason="reference CPU build (oracle/_ref) not present")
def test_cfg0_greedy_32_steps_bit_exact_against_reference():
    """Configuration 0 (28 layers, 151936-entry tied head) on the bench's
    prompt (128 ids, seed 1234): 32 free-running greedy ids equal the
    reference build's, and the logits that chose each equal it bit for bit;
    the device-resident greedy loop picks the same ids."""
    path = helpers.model_path(dict(sheep_b200.CONFIGS["qwen2.5-1.5b-q4"]))
    prompt = np.random.default_rng(1234).integers(0, 151936, 128).astype(np.int32)
    want_ids, want_lg = helpers.ref("decode", path, prompt=prompt, ngen=32, n_ctx=256, threads=16)
    eng = sheep_b200.Engine(path, n_ctx=256)
    try:
        ids, lgs = _cfg0_run(eng, prompt, 32)
        dev_ids = eng.generate(prompt, 32)
    finally:
        eng.close()
    assert np.array_equal(ids, want_ids), (ids, want_ids)
    assert _first_diff(lgs, want_lg) is None, _first_diff(lgs, want_lg)
    assert np.array_equal(dev_ids, want_ids)


@pytest.mark.skipif(not helpers.have_ref(), reason="reference CPU build (oracle/_ref) not present")
def test_llama8b_shapes_bit_exact_against_reference():
    """Configuration 3's widths (n_embd 4096, 32/8 heads, FFN 14336 -- the
    wide-row plan of the down projection --, vocab 128256, 6-bit group fields
    with negative mins) in two layers, teacher-forced: logits bit-equal to the
    reference build's."""
    spec = sheep_b200.spec_for("llama3-8b-q4k", n_layer=2)
    path = helpers.model_path(spec)
    toks = [int(t) for t in np.random.default_rng(21).integers(0, 128256, 10)]
    ref = helpers.ref("forward", path, tokens=toks, n_ctx=64, threads=8)
    eng = sheep_b200.Engine(path, n_ctx=64)
    try:
        got = np.array([eng.step(t, pos) for pos, t in enumerate(toks)])
    finally:
        eng.close()
    assert _first_diff(got, ref) is None, _first_diff(got, ref)
