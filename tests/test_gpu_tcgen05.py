"""The int8 tensor-core tile product (tcgen05.mma kind::i8, TMEM accumulator)
against exact integer matrix products: bit-exact."""
import numpy as np
import pytest

import sheep_b200

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def _imma(A, B):
    torch = _torch()
    M, K = A.shape
    N = B.shape[0]
    dA = torch.from_numpy(np.ascontiguousarray(A)).cuda()
    dB = torch.from_numpy(np.ascontiguousarray(B)).cuda()
    dC = torch.full((M, N), -7, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ok = sheep_b200.lib().sb_tc_imma(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), M, N, K, err.data_ptr(), None)
    assert ok, sheep_b200.lib().sb_tc_last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return dC.cpu().numpy()


@pytest.mark.parametrize("M,N,K", [(128, 16, 32), (128, 64, 256), (256, 32, 96), (128, 128, 512),
                                   (384, 256, 4096), (128, 16, 2048)])
def test_tc_imma_exact(M, N, K):
    rng = np.random.default_rng(M * 7 + N + K)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (N, K), dtype=np.int8)
    want = A.astype(np.int64) @ B.astype(np.int64).T
    got = _imma(A, B)
    assert np.array_equal(got.astype(np.int64), want)


def test_tc_imma_structured():
    """Identity-like operands locate every row and column: a wrong descriptor
    offset shows as a permuted result."""
    M, N, K = 128, 64, 256
    A = np.zeros((M, K), np.int8)
    B = np.zeros((N, K), np.int8)
    for r in range(M):
        A[r, (3 * r) % K] = 1
    for n in range(N):
        B[n, (3 * (2 * n)) % K] = 2
    want = A.astype(np.int64) @ B.astype(np.int64).T
    assert np.array_equal(_imma(A, B).astype(np.int64), want)


def test_tc_imma_rejects_bad_shapes():
    torch = _torch()
    A = torch.zeros((128, 64), dtype=torch.int8, device="cuda")
    C = torch.zeros((128, 24), dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    L = sheep_b200.lib()
    assert not L.sb_tc_imma(A.data_ptr(), A.data_ptr(), C.data_ptr(), 128, 24, 64, err.data_ptr(), None)
    assert not L.sb_tc_imma(A.data_ptr(), A.data_ptr(), C.data_ptr(), 100, 16, 64, err.data_ptr(), None)
    assert not L.sb_tc_imma(A.data_ptr(), A.data_ptr(), C.data_ptr(), 128, 16, 48, err.data_ptr(), None)


# ---------------------------------------------------------------- the batched path

from tests import helpers  # noqa: E402


def _width_model(nb, six):
    spec = sheep_b200.spec_for("tiny-q4", n_embd=512, n_ff=1408, n_head=8, n_head_kv=2, head_dim=64,
                               nbits=nb, emb_nbits=nb, scale6=six, minneg=six, n_layer=1, seed=100 + nb)
    return helpers.model_path(spec)


WIDTHS = [(4, 0), (8, 0), (6, 1), (2, 1), (3, 0), (5, 1), (7, 0), (4, 1)]


@pytest.mark.parametrize("nb,six", WIDTHS)
def test_requant8_bitexact(nb, six):
    """The int8 re-quantization (bound, scale, rounded fused weight) equals the
    CPU restatement of sml_g_requant8 bit for bit."""
    path = _width_model(nb, six)
    ts = sheep_b200.TensorSet(path)
    orc = helpers.Oracle(path)
    try:
        for name in ("blk.0.ffn_down.weight", "blk.0.attn_q.weight", "output.weight"):
            rows, cols, _ = ts.shape(name)
            w8, s8 = ts.requant8(name)
            ow8, os8 = orc.requant8(name, rows, cols)
            assert np.array_equal(w8, ow8), name
            assert np.array_equal(s8.view(np.uint32), os8.view(np.uint32)), name
    finally:
        ts.close()
        orc.close()


@pytest.mark.parametrize("nb,six", WIDTHS)
def test_gemm_tc_matches_restatement(nb, six):
    """The tensor-core product equals the CPU restatement of the batched path
    bit for bit (same int32 superblock dots, same fused epilogue in the same
    order), at 16 to 100 rows of x; and it stays within 2e-2 rel-RMS of the
    exact per-group product (measured 1.1-1.3e-2 on every width: the int8 weight
    step is 1/127 of the superblock's largest weight, and x is quantized per 256
    instead of per 32)."""
    path = _width_model(nb, six)
    ts = sheep_b200.TensorSet(path)
    orc = helpers.Oracle(path)
    rng = np.random.default_rng(nb * 11 + six)
    try:
        for name in ("blk.0.ffn_down.weight", "blk.0.attn_q.weight", "output.weight"):
            rows, cols, _ = ts.shape(name)
            for T in (16, 20, 64, 100):
                X = rng.standard_normal((T, cols)).astype(np.float16).astype(np.float32)
                Y = ts.gemm_tc(name, X)
                Yo = orc.gemm_sb(name, X, rows)
                assert np.array_equal(Y.view(np.uint32), Yo.view(np.uint32)), (name, T)
            worst = max(helpers.rel_rms(orc.matvec(name, X[t], rows), Y[t]) for t in range(0, T, 9))
            print(f"{name} Q{nb}{'f6' if six else 'f8'}: batched vs exact rel-RMS {worst:.2e}")
            assert worst <= 2e-2, worst
    finally:
        ts.close()
        orc.close()


def test_gemm_tc_cfg1_shapes():
    """Configuration 1's Q4 matrices (4096x4096, 14336x4096, 4096x14336) at 16
    and 64 rows of x, bit-equal to the restatement."""
    path = helpers.model_path(sheep_b200.spec_for("gemv-4096-q4"))
    ts = sheep_b200.TensorSet(path)
    orc = helpers.Oracle(path)
    rng = np.random.default_rng(23)
    try:
        for name in ("blk.0.attn_q.weight", "blk.0.ffn_gate.weight", "blk.0.ffn_down.weight"):
            rows, cols, _ = ts.shape(name)
            for T in (16, 64):
                X = rng.standard_normal((T, cols)).astype(np.float16).astype(np.float32)
                Y = ts.gemm_tc(name, X)
                Yo = orc.gemm_sb(name, X, rows)
                assert np.array_equal(Y.view(np.uint32), Yo.view(np.uint32)), (name, T)
    finally:
        ts.close()
        orc.close()
