"""The CPU oracle (oracle/sml_oracle.c) pinned against golden vectors that the
reference's own CPU code wrote (tests/golden/make_golden.py), and the
synthetic-model writer pinned by the files' sha256. No GPU.
"""
import json
import os

import numpy as np
import pytest

from tests import helpers

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
INDEX = json.load(open(os.path.join(GOLD, "index.json")))
WIDTH_FIXTURES = sorted(k for k in INDEX if k.startswith("width_"))


def check_input(n):
    i = np.arange(n, dtype=np.float32)
    return (np.sin(np.float32(0.001) * i) * (np.float32(1.0) + np.float32(0.5) * (i % 7).astype(np.float32))).astype(np.float32)


@pytest.mark.parametrize("fx", WIDTH_FIXTURES)
def test_writer_is_pinned(fx):
    path = helpers.model_path(INDEX[fx]["spec"])
    assert helpers.file_sha(path) == INDEX[fx]["sha256"]


@pytest.mark.parametrize("fx", WIDTH_FIXTURES)
def test_oracle_against_reference_vectors(fx):
    g = np.load(os.path.join(GOLD, fx))
    path = helpers.model_path(INDEX[fx]["spec"])
    recs = helpers.read_records(path)
    orc = helpers.Oracle(path, n_ctx=64)
    try:
        for t in ("blk.0.ffn_down.weight", "output.weight"):
            key = t.replace(".", "_")
            rows, cols = recs[t]["rows"], recs[t]["cols"]
            x = check_input(cols)
            # activation: gather through the tensor's perm, quantize -- bit-exact
            q, s, sums = helpers.oracle_quant(x[helpers.read_perm(path, t)])
            assert np.array_equal(q, g[key + "_q"])
            assert np.array_equal(s.view(np.uint32), g[key + "_s"].view(np.uint32))
            assert np.array_equal(sums, g[key + "_sums"])
            # the GEMV: the same integer dots and the reference's float order
            # for each width's kernels -- bit-exact
            y = orc.matvec(t, x, rows)
            assert np.array_equal(y.view(np.uint32), g[key + "_y"].view(np.uint32)), t
        r = recs["token_embd.weight"]
        for i, row in enumerate(g["embd_rows"]):
            d = orc.dequant_row("token_embd.weight", int(row), r["cols"])
            assert np.array_equal(d.view(np.uint32), g["embd_deq"][i].view(np.uint32))
    finally:
        orc.close()


def test_oracle_decode_against_reference():
    """The restatement's dense decode against the reference's own: 8 greedy
    ids after an 8-token prompt, logits equal bit for bit."""
    g = np.load(os.path.join(GOLD, "decode_tiny.npz"))
    path = helpers.model_path(INDEX["decode_tiny.npz"]["spec"])
    assert helpers.file_sha(path) == INDEX["decode_tiny.npz"]["sha256"]
    orc = helpers.Oracle(path, n_ctx=64)
    try:
        ids, lg = orc.decode(g["prompt"], 8)
    finally:
        orc.close()
    assert np.array_equal(ids, g["ids"])
    # every logit of every step, bit for bit: the restatement keeps the
    # reference's float order (matvec chains, attention, SiLU's exp, RoPE)
    assert np.array_equal(lg.view(np.uint32), g["logits"].view(np.uint32))


def test_quantize_edge_cases():
    """sml_quantize_act's rules on hand-made groups: zero group, exact .5 ties
    (round half to even), saturation at +-127, sums."""
    x = np.zeros(128, np.float32)
    x[32:64] = np.arange(32, dtype=np.float32) - 16.0          # amax 16: codes = rint(v * 127/16)
    x[64:96] = 127.0
    x[64] = -127.0
    x[96:128] = np.float32(0.5) * np.arange(32, dtype=np.float32)
    q, s, sums = helpers.oracle_quant(x)
    assert (q[:32] == 0).all() and s[0] == 0.0 and sums[0] == 0
    assert s[1] == np.float32(16.0) / np.float32(127.0)
    assert q[64] == -127 and (q[65:96] == 127).all()
    assert sums[2] == 31 * 127 - 127
    assert int(q[32:64].astype(np.int32).sum()) == int(sums[1])


def test_moe_route_matches_reference():
    rng = np.random.default_rng(12)
    for trial in range(20):
        lg = rng.standard_normal(128).astype(np.float32)
        if trial % 4 == 0:
            lg[rng.integers(0, 128, 8)] = lg.max()      # ties: the lower index wins
        sel, w = helpers.oracle_route(lg, 8, 1)
        order = sorted(range(128), key=lambda e: (-lg[e], e))[:8]
        assert list(sel) == order
        e = np.exp((lg[sel] - lg[sel[0]]).astype(np.float64))
        assert np.allclose(w, e / e.sum(), rtol=1e-6)
        if helpers.have_ref():
            rs, rw = helpers.ref("route", lg=lg, k=8, flags=1)
            assert np.array_equal(rs, sel) and np.array_equal(rw.view(np.uint32), w.view(np.uint32))


def test_oracle_moe_decode_against_reference():
    """The restatement's MoE branch (router, routing, experts, combine) against
    the reference's own decode of a two-layer, 16-expert model."""
    g = np.load(os.path.join(GOLD, "decode_moe_tiny.npz"))
    path = helpers.model_path(INDEX["decode_moe_tiny.npz"]["spec"])
    assert helpers.file_sha(path) == INDEX["decode_moe_tiny.npz"]["sha256"]
    orc = helpers.Oracle(path, n_ctx=64)
    try:
        ids, lg = orc.decode(g["prompt"], 8)
    finally:
        orc.close()
    assert np.array_equal(ids, g["ids"])
    # every logit of every step, bit for bit: the restatement keeps the
    # reference's float order (matvec chains, attention, SiLU's exp, RoPE)
    assert np.array_equal(lg.view(np.uint32), g["logits"].view(np.uint32))


def test_oracle_route_against_reference_vectors():
    """Choices bit-exact and weights bit-exact against sml_moe_route's outputs
    (both flags; ties, and a row where every expert ties)."""
    g = np.load(os.path.join(GOLD, "route.npz"))
    for flags in (1, 0):
        for t, lg in enumerate(g["logits"]):
            sel, w = helpers.oracle_route(lg, 8, flags)
            assert np.array_equal(sel, g[f"sel_f{flags}"][t]), (flags, t)
            assert np.array_equal(w.view(np.uint32), g[f"w_f{flags}"][t].view(np.uint32)), (flags, t)
    assert list(g["sel_f1"][1]) == list(range(8))


def test_oracle_batch_bookkeeping():
    """The batched restatement keeps one cache per slot: in the decode
    arithmetic (mode 0), ragged slots equal each sequence decoded alone, bit
    for bit; the batched arithmetic (mode 1) stays near them."""
    path = helpers.model_path(INDEX["decode_tiny.npz"]["spec"])
    rng = np.random.default_rng(3)
    ns, steps = 3, 7
    starts = [0, 2, 3]
    toks = rng.integers(0, 256, (ns, steps)).astype(np.int32)
    orc = helpers.Oracle(path, n_ctx=32)
    try:
        ob0 = helpers.OracleBatch(orc, ns, 0)
        ob1 = helpers.OracleBatch(orc, ns, 1, [1, 2, 1, 2, 1])
        got0, got1 = {}, {}
        for t in range(steps):
            pos = np.array([t - s if t >= s else -1 for s in starts], np.int32)
            tok = np.array([toks[s, max(p, 0)] for s, p in enumerate(pos)], np.int32)
            l0, l1 = ob0.step(tok, pos), ob1.step(tok, pos)
            for s in range(ns):
                if pos[s] >= 0:
                    got0[(s, pos[s])] = l0[s].copy()
                    got1[(s, pos[s])] = l1[s].copy()
        ob0.close()
        ob1.close()
        for s in range(ns):
            for p in range(steps - starts[s]):
                solo = orc.forward(int(toks[s, p]), p)   # the model's own cache, re-filled per sequence
                assert np.array_equal(solo.view(np.uint32), got0[(s, p)].view(np.uint32)), (s, p)
                assert helpers.rel_rms(solo, got1[(s, p)]) <= 6e-2
            # the next sequence re-uses positions 0.. of the model's cache
    finally:
        orc.close()


def test_quantize_act_sb_against_reference_vectors():
    """The batched path's per-256 activation (sml_quantize_act_sb) against the
    reference's own outputs: codes, per-group scales and sums bit for bit,
    including a zero superblock, .5 ties, one huge value, tiny values and a
    partial last superblock."""
    g = np.load(os.path.join(GOLD, "act_sb.npz"))
    for i in range(INDEX["act_sb.npz"]["inputs"]):
        q, s, sums = helpers.oracle_quant_sb(g[f"x{i}"])
        assert np.array_equal(q, g[f"q{i}"]), i
        assert np.array_equal(s.view(np.uint32), g[f"s{i}"].view(np.uint32)), i
        assert np.array_equal(sums, g[f"sums{i}"]), i


@pytest.mark.skipif(not helpers.have_ref(), reason="reference CPU build (oracle/_ref) not present")
def test_oracle_batch_equals_reference_forward_multi():
    """The restatement's multi-sequence step in the decode arithmetic (mode 0)
    against the reference's sml_forward_multi with SML_MULTI=exact (each
    conversation through the decode kernels, sml/sml-run.c:2579-2597):
    ragged starts, idle slots, five conversations -- logits bit for bit."""
    path = helpers.model_path(INDEX["decode_tiny.npz"]["spec"])
    ns, nsteps, starts = 5, 9, [0, 1, 2, 0, 4]
    toks = np.random.default_rng(3).integers(0, 1024, (nsteps, ns)).astype(np.int32)
    steps = [(toks[t].tolist(), [t - s if t >= s else -1 for s in starts]) for t in range(nsteps)]
    ref = helpers.ref("multi", path, ns=ns, n_vocab=1024, steps=steps, n_ctx=32, env={"SML_MULTI": "exact"})
    orc = helpers.Oracle(path, n_ctx=32)
    ob0 = helpers.OracleBatch(orc, ns, 0)
    try:
        for t, (tok, pos) in enumerate(steps):
            lg = ob0.step(np.array(tok, np.int32), np.array(pos, np.int32))
            for s in range(ns):
                if pos[s] >= 0:
                    assert np.array_equal(lg[s].view(np.uint32), ref[t][s].view(np.uint32)), (t, s)
    finally:
        ob0.close()
        orc.close()
