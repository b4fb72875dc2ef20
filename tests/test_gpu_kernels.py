"""Kernel-level parity on the GPU, through the C ABI, against the CPU oracle.

Bit-exact: int8 activation codes, scales and sums from identical inputs;
dequantized weights (multiply and add rounded separately, as the CPU does);
the streaming GEMV's outputs (the same integer dots, the float epilogue in the
reference's accumulator order) against the oracle and the reference build.
Tolerance: the batched GEMV over several vectors (weights read once per 8
vectors; its epilogue sums per unit, in another order) rel-RMS <= 1e-5 -- the
reference's own kernel gate is 1e-4, sml/sml-gpu-bench.c:147-154.
"""
import numpy as np
import pytest

import sheep_b200
from tests import helpers

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-5


def _torch():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def _quant_cases():
    rng = np.random.default_rng(5)
    x = rng.standard_normal(4096).astype(np.float32)
    x[:32] = 0.0                                   # an all-zero group: s = 0, is = 0
    x[32:64] = np.linspace(-1, 1, 32, dtype=np.float32)
    x[64:96] = (np.arange(32) - 15.5).astype(np.float32) * (127.0 / 15.5)   # ties at .5 after scaling
    x[96:128] = 1e-30                               # subnormal-range scale
    x[128:160] = 3e38 * np.sign(rng.standard_normal(32)).astype(np.float32)
    return [x, rng.standard_normal(1536).astype(np.float32) * 40.0, rng.standard_normal(8960).astype(np.float32)]


@pytest.mark.parametrize("case", range(3))
def test_quantize_act_bitexact(case):
    torch = _torch()
    x = _quant_cases()[case]
    n = len(x)
    dx = torch.from_numpy(x).cuda()
    dq = torch.zeros(n, dtype=torch.int8, device="cuda")
    ds = torch.zeros(n // 32, dtype=torch.float32, device="cuda")
    dsum = torch.zeros(n // 32, dtype=torch.int32, device="cuda")
    L = sheep_b200.lib()
    assert L.sb_quantize_act(dx.data_ptr(), None, n, dq.data_ptr(), ds.data_ptr(), dsum.data_ptr(), None)
    torch.cuda.synchronize()
    q, s, sums = helpers.oracle_quant(x)
    assert np.array_equal(dq.cpu().numpy(), q)
    assert np.array_equal(ds.cpu().numpy().view(np.uint32), s.view(np.uint32))
    assert np.array_equal(dsum.cpu().numpy(), sums)
    if helpers.have_ref():
        rq, rs, rsum = helpers.ref("quant", x=x)
        assert np.array_equal(rq, q) and np.array_equal(rs.view(np.uint32), s.view(np.uint32))
        assert np.array_equal(rsum, sums)


WIDTHS = [(nb, six) for six in (0, 1) for nb in (2, 3, 4, 5, 6, 7, 8)]


def _width_model(nb, six):
    spec = sheep_b200.spec_for("tiny-q4", n_embd=512, n_ff=1408, n_head=8, n_head_kv=2, head_dim=64,
                               nbits=nb, emb_nbits=nb, scale6=six, minneg=six, n_layer=1, seed=100 + nb)
    return helpers.model_path(spec)


@pytest.mark.parametrize("nb,six", WIDTHS)
def test_gemv_all_widths(nb, six):
    path = _width_model(nb, six)
    ts = sheep_b200.TensorSet(path)
    orc = helpers.Oracle(path)
    rng = np.random.default_rng(nb * 10 + six)
    try:
        for name in ("blk.0.attn_q.weight", "blk.0.ffn_down.weight", "blk.0.ffn_gate.weight", "output.weight"):
            rows, cols, got_nb = ts.shape(name)
            assert got_nb == nb
            x = rng.standard_normal(cols).astype(np.float32)
            y, q, s, sums = ts.matvec(name, x)
            yo = orc.matvec(name, x, rows)
            assert np.array_equal(y.view(np.uint32), yo.view(np.uint32)), name
            # the activation the kernel quantized: bit-exact against the CPU's
            perm = helpers.read_perm(path, name)
            oq, os_, osum = helpers.oracle_quant(x[perm])
            assert np.array_equal(q, oq) and np.array_equal(s.view(np.uint32), os_.view(np.uint32))
            assert np.array_equal(sums, osum)
    finally:
        ts.close()
        orc.close()


@pytest.mark.parametrize("nb,six", WIDTHS)
def test_dequant_rows_bitexact(nb, six):
    path = _width_model(nb, six)
    ts = sheep_b200.TensorSet(path)
    orc = helpers.Oracle(path)
    try:
        name = "token_embd.weight"
        rows, cols, _ = ts.shape(name)
        pick = [0, 1, 7, rows // 2, rows - 1]
        got = ts.dequant_rows(name, pick)
        for i, r in enumerate(pick):
            want = orc.dequant_row(name, r, cols)
            assert np.array_equal(got[i].view(np.uint32), want.view(np.uint32)), (name, r)
    finally:
        ts.close()
        orc.close()


@pytest.mark.skipif(not helpers.have_ref(), reason="reference CPU build (oracle/_ref) not present")
@pytest.mark.parametrize("nb,six", [(4, 0), (8, 0), (6, 1), (4, 1), (3, 0)])
def test_gemv_against_reference_build(nb, six):
    """The same GEMV against the reference's own kernels (oracle/_ref)."""
    path = _width_model(nb, six)
    ts = sheep_b200.TensorSet(path)
    try:
        rng = np.random.default_rng(77)
        for name in ("blk.0.attn_q.weight", "blk.0.ffn_down.weight"):
            rows, cols, _ = ts.shape(name)
            x = rng.standard_normal(cols).astype(np.float32)
            y, q, s, sums = ts.matvec(name, x)
            ry, rq, rs, rsum = helpers.ref("matvec", path, name=name, x=x, rows=rows)
            assert np.array_equal(q, rq) and np.array_equal(sums, rsum)
            assert np.array_equal(y.view(np.uint32), ry.view(np.uint32)), name
    finally:
        ts.close()


def _cfg0_layer_model():
    # one layer at the config-0 widths with a 32768-row head: tensors tile at
    # TR = 1..8 with many tiles per CTA, so every ring stage is reused
    spec = sheep_b200.spec_for("qwen2.5-1.5b-q4", n_layer=1, n_vocab=32768, tied=0, seed=21)
    return helpers.model_path(spec)


def test_gemv_cfg0_shapes_stage_reuse():
    path = _cfg0_layer_model()
    ts = sheep_b200.TensorSet(path)
    orc = helpers.Oracle(path)
    rng = np.random.default_rng(99)
    try:
        for name in ("blk.0.attn_q.weight", "blk.0.attn_k.weight", "blk.0.ffn_gate.weight",
                     "blk.0.ffn_down.weight", "output.weight"):
            rows, cols, _ = ts.shape(name)
            x = rng.standard_normal(cols).astype(np.float32)
            y, q, s, sums = ts.matvec(name, x)
            assert np.array_equal(y.view(np.uint32), orc.matvec(name, x, rows).view(np.uint32)), name
            # repeated calls are bit-identical (no dependence on timing)
            y2, _, _, _ = ts.matvec(name, x)
            assert np.array_equal(y.view(np.uint32), y2.view(np.uint32)), name
    finally:
        ts.close()
        orc.close()


@pytest.mark.parametrize("n_ff", [8960, 1408])
def test_gemv_prepermuted_staging_bitexact(n_ff):
    """The pre-permuted staging: the input already in the tensor's column
    order, quantized one lane per group (no gather), as the tensor-parallel
    down projection stages it and as the one-GPU gate/up GEMV quantizes the
    hidden vector for down (the same quant_lanes code; that path is checked
    end to end by the decode tests' bit-exact logits). On
    configuration 0's 8960-column input and on 1408 columns (44 groups: not a
    multiple of the 512 consumer threads' groups): the exported codes, scales
    and sums equal the per-32 quantization of the same values, bit for bit,
    through an all-zero group, exact .5 ties, saturation and huge values; the
    GEMV equals the oracle's on the same x."""
    spec = sheep_b200.spec_for("tiny-q4", n_embd=512, n_ff=n_ff, n_head=8, n_head_kv=2, head_dim=64,
                               n_layer=1, seed=123)
    path = helpers.model_path(spec)
    ts = sheep_b200.TensorSet(path)
    orc = helpers.Oracle(path)
    try:
        name = "blk.0.ffn_down.weight"
        rows, cols, _ = ts.shape(name)
        perm = helpers.read_perm(path, name)
        rng = np.random.default_rng(n_ff)
        for case in range(3):
            xp = rng.standard_normal(cols).astype(np.float32) * (1.0, 40.0, 1e-3)[case]
            xp[:32] = 0.0                                                    # zero group
            xp[32:64] = (np.arange(32) - 15.5).astype(np.float32) * (127.0 / 15.5)   # .5 ties
            xp[-32:] = rng.standard_normal(32).astype(np.float32) * 1e-30            # tiny scale
            huge = xp.copy()
            huge[64:96] = 3e38 * np.sign(rng.standard_normal(32)).astype(np.float32)  # saturation (y overflows)
            for v in (huge, xp):
                _, q, s, sums = ts.matvec(name, v, permuted=True)
                oq, os_, osum = helpers.oracle_quant(v)
                assert np.array_equal(q, oq), case
                assert np.array_equal(s.view(np.uint32), os_.view(np.uint32)), case
                assert np.array_equal(sums, osum), case
            y, _, _, _ = ts.matvec(name, xp, permuted=True)
            x = np.zeros_like(xp)
            x[perm] = xp                                                     # the same values, natural order
            yo = orc.matvec(name, x, rows)
            assert np.array_equal(y.view(np.uint32), yo.view(np.uint32)), case
    finally:
        ts.close()
        orc.close()


# ------------------------------------------------------------------ decode attention

def _attn_reference(qkv, kc, vc, cos, sin, nh, nkv, hd, pos, scale, qn=None, kn=None, eps=1e-6):
    """RoPE by halved pairs, fp16 cache rounding, softmax attention in float64
    (sml/sml-run.c:180-266, 339-375)."""
    q = qkv[:nh * hd].reshape(nh, hd).astype(np.float64)
    k = qkv[nh * hd:(nh + nkv) * hd].reshape(nkv, hd).astype(np.float64)
    v = qkv[(nh + nkv) * hd:].reshape(nkv, hd).astype(np.float64)
    if qn is not None:
        q = q / np.sqrt((q * q).mean(1, keepdims=True) + eps) * qn
        k = k / np.sqrt((k * k).mean(1, keepdims=True) + eps) * kn
    half = hd // 2

    def rope(x):
        a, b = x[:, :half], x[:, half:]
        c, s = cos[pos].astype(np.float64), sin[pos].astype(np.float64)
        return np.concatenate([a * c - b * s, a * s + b * c], 1)

    q, k = rope(q), rope(k)
    k16, v16 = k.astype(np.float16), v.astype(np.float16)
    K = kc[:pos + 1].reshape(pos + 1, nkv, hd).astype(np.float64)
    V = vc[:pos + 1].reshape(pos + 1, nkv, hd).astype(np.float64)
    K[pos], V[pos] = k16, v16
    rep = nh // nkv
    out = np.zeros((nh, hd))
    for h in range(nh):
        s = K[:, h // rep] @ q[h] * scale
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ V[:, h // rep]
    return out.reshape(-1), k16, v16


@pytest.mark.parametrize("hd,nh,nkv,pos,norm", [(128, 12, 2, 0, False), (128, 12, 2, 37, False),
                                                 (128, 12, 2, 64, False), (128, 12, 2, 200, False),
                                                 (64, 8, 2, 130, True), (128, 32, 8, 255, False)])
def test_attention_decode(hd, nh, nkv, pos, norm):
    torch = _torch()
    rng = np.random.default_rng(pos + hd)
    n_ctx = 256
    qkv = rng.standard_normal((nh + 2 * nkv) * hd).astype(np.float32)
    kc = rng.standard_normal((n_ctx, nkv * hd)).astype(np.float16)
    vc = rng.standard_normal((n_ctx, nkv * hd)).astype(np.float16)
    i = np.arange(hd // 2, dtype=np.float32)
    freq = np.float32(1e6) ** (-i / np.float32(hd // 2))
    ang = np.arange(n_ctx, dtype=np.float32)[:, None] * freq[None, :]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    qn = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32) if norm else None
    kn = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32) if norm else None
    scale = 1.0 / np.sqrt(hd)
    want, k16, v16 = _attn_reference(qkv, kc, vc, cos, sin, nh, nkv, hd, pos, scale, qn, kn)
    d = {n: torch.from_numpy(np.ascontiguousarray(a)).cuda() for n, a in
         dict(qkv=qkv, kc=kc.view(np.uint16), vc=vc.view(np.uint16), cos=cos, sin=sin).items()}
    dn = {n: (torch.from_numpy(a).cuda() if a is not None else None) for n, a in dict(qn=qn, kn=kn).items()}
    out = torch.zeros(nh * hd, dtype=torch.float32, device="cuda")
    L = sheep_b200.lib()
    ok = L.sb_attn_decode(d["qkv"].data_ptr(), d["kc"].data_ptr(), d["vc"].data_ptr(), d["cos"].data_ptr(),
                          d["sin"].data_ptr(), dn["qn"].data_ptr() if norm else None,
                          dn["kn"].data_ptr() if norm else None, 1e-6, nh, nkv, hd, n_ctx, pos, float(scale),
                          out.data_ptr(), None)
    assert ok, L.sb_attn_last_error()
    got = out.cpu().numpy()
    assert helpers.rel_rms(want, got) <= 1e-5
    # the cache row at pos: the roped key and the value, fp16 (last-bit ties allowed)
    kw = d["kc"].cpu().numpy().view(np.float16)[pos].reshape(nkv, hd)
    vw = d["vc"].cpu().numpy().view(np.float16)[pos].reshape(nkv, hd)
    assert np.array_equal(vw, v16)
    assert np.abs(kw.astype(np.float64) - k16.astype(np.float64)).max() <= \
        np.abs(k16.astype(np.float64)).max() * 2.0 ** -10
    # positions other than pos untouched
    assert np.array_equal(d["kc"].cpu().numpy()[:pos], kc.view(np.uint16)[:pos])


@pytest.mark.parametrize("nb,six", [(4, 0), (8, 0), (6, 1), (2, 1), (3, 0), (5, 1), (7, 0)])
def test_batched_gemv_widths(nb, six):
    """The batched GEMV (weights read once per 8 vectors) against the oracle
    vector by vector, at batches of 1 (the streaming GEMV), 4, 13 and 16."""
    path = _width_model(nb, six)
    ts = sheep_b200.TensorSet(path)
    orc = helpers.Oracle(path)
    rng = np.random.default_rng(nb * 7 + six)
    try:
        for name in ("blk.0.ffn_down.weight", "blk.0.attn_q.weight"):
            rows, cols, _ = ts.shape(name)
            for B in (1, 4, 13, 16):
                X = rng.standard_normal((B, cols)).astype(np.float16).astype(np.float32)
                Y = ts.gemv(name, X)
                for b in range(B):
                    yo = orc.matvec(name, X[b], rows)
                    if B == 1:
                        assert np.array_equal(Y[b].view(np.uint32), yo.view(np.uint32)), name
                    assert helpers.rel_rms(yo, Y[b]) <= GEMV_TOL, (name, B, b)
    finally:
        ts.close()
        orc.close()


@pytest.mark.parametrize("cfg", ["gemv-4096-q4", "gemv-4096-q8"])
def test_gemv_microbench_shapes(cfg):
    """Configuration 1's matrices (4096x4096, 14336x4096, 4096x14336; Q4 and
    Q8) at batches 1, 4 and 16. The 14336-column rows do not leave room for the
    input copy and a 16-stage ring: they run with the input gathered from L2
    and a shorter ring."""
    path = helpers.model_path(sheep_b200.spec_for(cfg))
    ts = sheep_b200.TensorSet(path)
    orc = helpers.Oracle(path)
    rng = np.random.default_rng(17)
    try:
        for name in ("blk.0.attn_q.weight", "blk.0.ffn_gate.weight", "blk.0.ffn_down.weight"):
            rows, cols, _ = ts.shape(name)
            for B in (1, 4, 16):
                X = rng.standard_normal((B, cols)).astype(np.float16).astype(np.float32)
                Y = ts.gemv(name, X)
                for b in range(0, B, 3):
                    yo = orc.matvec(name, X[b], rows)
                    if B == 1:
                        assert np.array_equal(Y[b].view(np.uint32), yo.view(np.uint32)), name
                    assert helpers.rel_rms(yo, Y[b]) <= GEMV_TOL, (name, B, b)
    finally:
        ts.close()
        orc.close()
