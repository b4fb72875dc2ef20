"""The mixture-of-experts FFN on the GPU against the CPU oracle.

Routing: the chosen experts bit-exact (sml_moe_route's top-k, ties to the lower
index). The decode path (one token a step) runs the reference's float order
end to end -- the router's double sums, the libm expf of the weights, each
expert's matvec chains and SiLU, the combine's fused multiply-adds -- so a MoE
decoder's logits equal the reference's bit for bit, and so does the layer at
one token a step. With several tokens a step an expert's tile is read once for
up to eight tokens and each lane sums its share of the float epilogue
(another order than the reference's): the same experts, outputs within
rel-RMS 3e-3 of the oracle's (a hidden value at a rounding boundary of its
int8 code meets the down projection one code away, about 1e-3 of the output
for one such flip). Rows without a flip agree to 1e-4, and at 16 or more rows
most rows must. The routing entry point alone (no libm table) rounds exp from
double: weights within 2e-6 relative.
"""
import json
import os

import numpy as np
import pytest

import sheep_b200
from tests import helpers

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
INDEX = json.load(open(os.path.join(GOLD, "index.json")))
Y_RELRMS = 3e-3          # a few int8 code flips in the hidden vector
Y_RELRMS_CLEAN = 1e-4    # a row without one
W_RTOL = 2e-6


def _torch():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def _rows(seed, T, E):
    """fp16 N(0, 1) token rows as the layer's float input."""
    return np.random.default_rng(seed).standard_normal((T, E)).astype(np.float16).astype(np.float32)


def _route_dev(lg, k, flags):
    torch = _torch()
    d = torch.from_numpy(np.ascontiguousarray(lg, np.float32)).cuda()
    T, ne = lg.shape
    sel = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
    w = torch.zeros((T, k), dtype=torch.float32, device="cuda")
    sheep_b200.moe_route_dev(d.data_ptr(), T, ne, k, flags, sel.data_ptr(), w.data_ptr())
    torch.cuda.synchronize()
    return sel.cpu().numpy(), w.cpu().numpy()


def test_route_against_reference_vectors():
    g = np.load(os.path.join(GOLD, "route.npz"))
    for flags in (1, 0):
        sel, w = _route_dev(g["logits"], 8, flags)
        assert np.array_equal(sel, g[f"sel_f{flags}"]), flags
        assert np.allclose(w, g[f"w_f{flags}"], rtol=W_RTOL, atol=0), flags


@pytest.mark.parametrize("ne,k", [(128, 8), (256, 16), (60, 6), (8, 8), (1, 1)])
def test_route_against_oracle(ne, k):
    rng = np.random.default_rng(ne * 31 + k)
    lg = rng.standard_normal((300, ne)).astype(np.float32)
    lg[::7, rng.integers(0, ne, 3)] = lg[::7].max(axis=1, keepdims=True)   # planted ties
    lg[5::11] = np.float32(-1.25)                                          # all tied
    for flags in (1, 0):
        sel, w = _route_dev(lg, k, flags)
        for t in range(len(lg)):
            s, ww = helpers.oracle_route(lg[t], k, flags)
            assert np.array_equal(sel[t], s), (flags, t)
            assert np.allclose(w[t], ww, rtol=W_RTOL, atol=0), (flags, t)


def test_route_rejects_bad_arguments():
    torch = _torch()
    d = torch.zeros((4, 300), dtype=torch.float32, device="cuda")
    sel = torch.zeros((4, 8), dtype=torch.int32, device="cuda")
    w = torch.zeros((4, 8), dtype=torch.float32, device="cuda")
    for ne, k, flags in ((300, 8, 1), (128, 17, 1), (128, 0, 1), (128, 8, 2)):
        with pytest.raises(RuntimeError):
            sheep_b200.moe_route_dev(d.data_ptr(), 4, ne, k, flags, sel.data_ptr(), w.data_ptr())


def _check_layer(path, T, seed, layer=0):
    """The integer kernels (tensor cores off) against the oracle."""
    m = sheep_b200.MoeLayer(path, layer=layer, max_tokens=max(T, 1))
    m.tensor_cores(False)
    orc = helpers.Oracle(path, n_ctx=64)
    try:
        x = _rows(seed, T, m.n_embd)
        y, sel, w, n_active = m.forward(x)
        yo, so, wo = orc.moe_ffn(layer, x)
        assert np.array_equal(sel, so)
        assert np.allclose(w, wo, rtol=W_RTOL, atol=0)
        assert n_active == len(np.unique(so))
        if T == 1:
            # one token a step: the decode path, the reference's float order
            assert np.array_equal(w.view(np.uint32), wo.view(np.uint32))
            assert np.array_equal(y.view(np.uint32), yo.view(np.uint32))
            return y
        errs = np.array([helpers.rel_rms(yo[t], y[t]) for t in range(T)])
        assert errs.max() <= Y_RELRMS, errs.max()
        if T >= 16:
            assert np.mean(errs <= Y_RELRMS_CLEAN) >= 0.75, np.sort(errs)[-8:]
        return y
    finally:
        m.close()
        orc.close()


def test_layer_cfg2_shape():
    """The Qwen3-30B-A3B-shaped layer (2048 wide, 128 experts, top 8, FFN 768)
    at 1, 16, 64 and 256 tokens a step: one token per chunk at T = 1, up to
    eight at once above."""
    path = helpers.model_path(sheep_b200.spec_for("qwen3-30b-a3b-moe-layer"))
    for T in (1, 16, 64, 256):
        _check_layer(path, T, seed=T)


@pytest.mark.parametrize("nb,six", [(nb, six) for six in (0, 1) for nb in (2, 3, 4, 5, 6, 7, 8)])
def test_layer_every_width(nb, six):
    spec = sheep_b200.spec_for("tiny-q4", n_layer=1, nbits=nb, scale6=six, minneg=six, n_expert=8,
                               n_expert_used=2, moe_flags=1, expert_ff=128, seed=700 + 10 * nb + six)
    path = helpers.model_path(spec)
    _check_layer(path, 1, seed=1)
    _check_layer(path, 13, seed=2)


def test_layer_softmax_over_all_experts():
    spec = sheep_b200.spec_for("tiny-q4", n_layer=1, n_expert=16, n_expert_used=4, moe_flags=0, expert_ff=256,
                               seed=41)
    _check_layer(helpers.model_path(spec), 9, seed=3)


def test_rows_do_not_depend_on_the_batch():
    """A row's output is the same whichever rows share its step (chunks of
    eight tokens per expert form differently)."""
    spec = sheep_b200.spec_for("tiny-q4", n_layer=1, n_expert=16, n_expert_used=4, moe_flags=1, expert_ff=256,
                               seed=42)
    path = helpers.model_path(spec)
    m = sheep_b200.MoeLayer(path, max_tokens=64)
    m.tensor_cores(False)
    try:
        x = _rows(5, 64, m.n_embd)
        a = m.forward(x[:16])[0]
        b = m.forward(x)[0][:16]
        c = m.forward(x[::-1].copy())[0][::-1][:16]
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert np.array_equal(a.view(np.uint32), c.view(np.uint32))
    finally:
        m.close()


# The tensor-core path (calls of 16+ rows): fp16 weights decoded from the
# four-bit codes, fp16 rows, fp32 sums. Checked against the layer computed
# exactly (float64 over the dequantized weights): per row within 3e-3 relative
# RMS (fp16 rounding of both operands and of the hidden vector). The decode
# arithmetic (int8 rows per 32 before each product, the reference's) is itself
# ~1e-2 from exact at these shapes, so the two paths differ by about that much.
TC_EXACT = 3e-3
TC_VS_DECODE = 3e-2


def _exact_layer(orc, path, x, sel, w, layer=0):
    """The MoE FFN in float64 over the oracle's dequantized weights: each
    chosen expert's SiLU(gate x) * (up x), its down product, weighted sum."""
    T, E = x.shape
    recs = helpers.read_records(path)
    y = np.zeros((T, E), np.float64)
    for e in np.unique(sel):
        g, u, d = (f"blk.{layer}.ffn_{n}.{e}.weight" for n in ("gate", "up", "down"))
        F = recs[g]["rows"]
        Wg = np.array([orc.dequant_row(g, r, E) for r in range(F)], np.float64)
        Wu = np.array([orc.dequant_row(u, r, E) for r in range(F)], np.float64)
        Wd = np.array([orc.dequant_row(d, r, F) for r in range(E)], np.float64)
        pg, pd = helpers.read_perm(path, g), helpers.read_perm(path, d)
        for t, j in zip(*np.nonzero(sel == e)):
            xg = x[t].astype(np.float64)[pg]          # column k of gate/up takes x[perm[k]]
            a, b = Wg @ xg, Wu @ xg
            h = a / (1.0 + np.exp(-a)) * b
            y[t] += float(w[t, j]) * (Wd @ h[pd])
    return y


def _check_tc(path, T, seed, exact=True):
    m = sheep_b200.MoeLayer(path, max_tokens=T)
    orc = helpers.Oracle(path, n_ctx=64)
    try:
        assert m.tensor_cores(True)
        x = _rows(seed, T, m.n_embd)
        y, sel, w, n_active = m.forward(x)
        m.tensor_cores(False)
        yi = m.forward(x)[0]
        yo, so, wo = orc.moe_ffn(0, x)
        assert np.array_equal(sel, so)
        assert np.allclose(w, wo, rtol=W_RTOL, atol=0)
        # the layer's input rows as the experts see them (no norm in sb_moe: x itself)
        errs_d = np.array([helpers.rel_rms(yo[t], y[t]) for t in range(T)])
        errs_i = np.array([helpers.rel_rms(yi[t], y[t]) for t in range(T)])
        print(f"T={T}: tensor cores vs decode arithmetic rel-RMS median {np.median(errs_d):.2e} max {errs_d.max():.2e}; "
              f"vs integer kernels max {errs_i.max():.2e}")
        assert errs_d.max() <= TC_VS_DECODE and errs_i.max() <= TC_VS_DECODE
        if exact:
            ye = _exact_layer(orc, path, x, sel, w)
            errs_e = np.array([helpers.rel_rms(ye[t], y[t]) for t in range(T)])
            errs_de = np.array([helpers.rel_rms(ye[t], yo[t]) for t in range(T)])
            print(f"T={T}: vs exact: tensor cores max {errs_e.max():.2e} median {np.median(errs_e):.2e}; "
                  f"decode arithmetic max {errs_de.max():.2e} median {np.median(errs_de):.2e}")
            assert errs_e.max() <= TC_EXACT, errs_e.max()
    finally:
        m.close()
        orc.close()


def test_layer_tensor_cores_cfg2_shape():
    """The Qwen3-30B-A3B-shaped layer at 16, 64 and 256 tokens a step on the
    tensor cores: the same routing, outputs within the stated tolerance of the
    oracle and of the integer kernels."""
    path = helpers.model_path(sheep_b200.spec_for("qwen3-30b-a3b-moe-layer"))
    for T in (16, 64, 256):
        _check_tc(path, T, seed=100 + T, exact=T == 16)


def test_layer_tensor_cores_split_chunks():
    """16 experts, top 4, 256 tokens: most experts get more than 64 rows, so
    their rows split over several chunks; also a call of exactly 16 rows."""
    spec = sheep_b200.spec_for("tiny-q4", n_layer=1, n_expert=16, n_expert_used=4, moe_flags=1, expert_ff=256,
                               seed=43)
    path = helpers.model_path(spec)
    _check_tc(path, 256, seed=6)
    _check_tc(path, 16, seed=7)


def test_layer_tensor_cores_rows_independent():
    """On the tensor cores too a row's output does not depend on the rows
    sharing its step (its column of the product is its own), bit for bit."""
    spec = sheep_b200.spec_for("tiny-q4", n_layer=1, n_expert=16, n_expert_used=4, moe_flags=1, expert_ff=256,
                               seed=44)
    path = helpers.model_path(spec)
    m = sheep_b200.MoeLayer(path, max_tokens=96)
    try:
        assert m.tensor_cores(True)
        x = _rows(8, 96, m.n_embd)
        a = m.forward(x[:16])[0]
        b = m.forward(x)[0][:16]
        c = m.forward(x[::-1].copy())[0][::-1][:16]
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert np.array_equal(a.view(np.uint32), c.view(np.uint32))
    finally:
        m.close()


def test_layer_rejects_bad_arguments():
    spec = sheep_b200.spec_for("tiny-q4", n_layer=1, n_expert=8, n_expert_used=2, moe_flags=1, expert_ff=128)
    path = helpers.model_path(spec)
    with pytest.raises(RuntimeError):
        sheep_b200.MoeLayer(path, layer=1)
    with pytest.raises(RuntimeError):
        sheep_b200.MoeLayer(helpers.model_path(sheep_b200.spec_for("tiny-q4")))   # dense: no router
    m = sheep_b200.MoeLayer(path, max_tokens=4)
    try:
        with pytest.raises(RuntimeError):
            m.forward(np.zeros((5, m.n_embd), np.float32))
    finally:
        m.close()


def test_moe_decode_against_oracle():
    """A two-layer, 16-expert MoE decoder through the engine: 40
    teacher-forced positions bit-equal to the oracle's logits; the
    reference's own 8 greedy steps (ids and every logit, bit for bit), then 32
    free-running greedy ids equal to the oracle's."""
    path = helpers.model_path(INDEX["decode_moe_tiny.npz"]["spec"])
    g = np.load(os.path.join(GOLD, "decode_moe_tiny.npz"))
    eng = sheep_b200.Engine(path, n_ctx=96)
    orc = helpers.Oracle(path, n_ctx=96)
    try:
        toks = np.random.default_rng(8).integers(0, 1024, 40)
        for pos, t in enumerate(toks):
            lg, lo = eng.step(int(t), pos), orc.forward(int(t), pos)
            assert np.array_equal(lg.view(np.uint32), lo.view(np.uint32)), \
                (pos, int((lg.view(np.uint32) != lo.view(np.uint32)).sum()))
    finally:
        eng.close()
        orc.close()
    eng = sheep_b200.Engine(path, n_ctx=96)
    try:
        lg = None
        for i, t in enumerate(g["prompt"]):
            lg = eng.step(int(t), i)
        for s in range(len(g["ids"])):
            assert np.array_equal(lg.view(np.uint32), g["logits"][s].view(np.uint32)), s
            t = int(np.argmax(lg))
            assert t == int(g["ids"][s]), s
            lg = eng.step(t, len(g["prompt"]) + s)
        ids32 = eng.generate(g["prompt"], 32)
    finally:
        eng.close()
    orc = helpers.Oracle(path, n_ctx=96)
    try:
        want, _ = orc.decode(g["prompt"], 32)
    finally:
        orc.close()
    assert np.array_equal(ids32, want)
