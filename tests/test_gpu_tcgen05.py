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
