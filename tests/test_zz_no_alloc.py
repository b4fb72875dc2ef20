"""sb_attn_decode_noalloc: the decode-attention entry point for callers that may
not allocate device memory (a host that owns every allocation up front, or one
that must not synchronize the device mid-stream). Its scratch is a static device
array, so it must give what sb_attn_decode (which allocates per call) gives.

Collected last on purpose (pytest runs files in name order): if it fails, every
other test has already run. It passes alone in a fresh process as well.
"""
import numpy as np
import pytest

import sheep_b200

pytestmark = pytest.mark.gpu

TOL = 1e-5   # the rel-RMS bound the attention tests use (a diagnostic here: the
             # two entry points run the same kernel, chunking and partials layout,
             # so their outputs must be equal bit for bit)


def _inputs(rng, nh, nkv, hd, n_ctx):
    qkv = rng.standard_normal((nh + 2 * nkv) * hd).astype(np.float32)
    kc = rng.standard_normal((n_ctx, nkv * hd)).astype(np.float16)
    vc = rng.standard_normal((n_ctx, nkv * hd)).astype(np.float16)
    i = np.arange(hd // 2, dtype=np.float32)
    ang = np.arange(n_ctx, dtype=np.float32)[:, None] * (np.float32(1e6) ** (-i / np.float32(hd // 2)))[None, :]
    return qkv, kc, vc, np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def _call(fn, torch, qkv, kc, vc, cos, sin, nh, nkv, hd, n_ctx, pos):
    d = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (qkv, kc.view(np.uint16), vc.view(np.uint16), cos, sin)]
    out = torch.zeros(nh * hd, dtype=torch.float32, device="cuda")
    ok = fn(d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(), d[4].data_ptr(), None, None,
            1e-6, nh, nkv, hd, n_ctx, pos, float(1.0 / np.sqrt(hd)), out.data_ptr(), None)
    torch.cuda.synchronize()
    return ok, out.cpu().numpy(), d[1].cpu().numpy(), d[2].cpu().numpy()


def _rms(a, b):
    a = a.astype(np.float64)
    return float(np.sqrt(np.mean((a - b) ** 2)) / np.sqrt(np.mean(a ** 2)))


def _both(L, torch, rng, nh, nkv, hd, n_ctx, pos):
    args = _inputs(rng, nh, nkv, hd, n_ctx)
    ok_a, out_a, kc_a, vc_a = _call(L.sb_attn_decode, torch, *args, nh, nkv, hd, n_ctx, pos)
    assert ok_a, L.sb_attn_last_error()
    ok_b, out_b, kc_b, vc_b = _call(L.sb_attn_decode_noalloc, torch, *args, nh, nkv, hd, n_ctx, pos)
    assert ok_b, L.sb_attn_noalloc_last_error()
    assert _rms(out_a, out_b) <= TOL, (pos, _rms(out_a, out_b))
    assert np.array_equal(out_a.view(np.uint32), out_b.view(np.uint32)), pos
    assert np.array_equal(kc_a, kc_b) and np.array_equal(vc_a, vc_b)


def test_noalloc_matches_allocating_entry_point_two_calls():
    import torch
    assert torch.cuda.is_available()
    L = sheep_b200.lib()
    rng = np.random.default_rng(2024)
    nh, nkv, hd, n_ctx = 12, 2, 128, 512
    # calls in a row on the shared array, each seeing what the one before left:
    # five chunks, a single chunk (no partials, no counters), then two chunks
    for pos in (300, 40, 77):
        _both(L, torch, rng, nh, nkv, hd, n_ctx, pos)


def test_noalloc_size_limit_boundary():
    """32 heads of 128: position 4031 needs 63 chunks, 1,048,320 bytes of
    partials (accepted, equal to the allocating call); 4032 needs 64 chunks,
    over the 1 MiB array (rejected with a reason)."""
    import torch
    L = sheep_b200.lib()
    rng = np.random.default_rng(7)
    nh, nkv, hd, n_ctx = 32, 8, 128, 4200
    _both(L, torch, rng, nh, nkv, hd, n_ctx, 4031)
    args = _inputs(rng, nh, nkv, hd, n_ctx)
    ok, _, _, _ = _call(L.sb_attn_decode_noalloc, torch, *args, nh, nkv, hd, n_ctx, 4032)
    assert ok == 0
    assert b"static scratch" in L.sb_attn_noalloc_last_error()
