"""The C ABI without a GPU: the library loads and exports every function that
include/*.h declares; the SSF loader's accept/reject behaviour on malformed
files (the categories of the reference's sml/sml-model-test.c:158-206),
checked against the reference loader when its build is present.
"""
import os
import re
import shutil
import struct
import tempfile

import pytest

import sheep_b200
from tests import helpers

ROOT = helpers.ROOT


def declared_functions():
    names = set()
    for h in ("sml-gpu.h", "sheep_b200.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"//.*", "", src)
        for m in re.finditer(r"\b([a-z_][a-z0-9_]*)\s*\(", src):
            name = m.group(1)
            if name.startswith(("sml_gpu_", "sb_", "ssfgen_")):
                names.add(name)
    return sorted(names)


def test_header_symbols_exported():
    import ctypes
    L = ctypes.CDLL(sheep_b200.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing
    assert len(declared_functions()) >= 25


def test_reference_api_declared():
    """The seven entry points of the reference's sml/sml-gpu.h, same names."""
    want = {"sml_gpu_open", "sml_gpu_prefill", "sml_gpu_step", "sml_gpu_layers", "sml_gpu_prompt_mode",
            "sml_gpu_decode_cpu", "sml_gpu_set_middle"}
    assert want <= set(declared_functions())


# ------------------------------------------------------------------ loader fixtures

HDR = 4096
REC = 248


def _valid_model():
    return helpers.model_path(sheep_b200.spec_for("tiny-q4", n_layer=1, seed=3))


def _mutate(fn):
    src = _valid_model()
    d = tempfile.mkdtemp()
    dst = os.path.join(d, "m.ssf")
    shutil.copy(src, dst)
    with open(dst, "r+b") as f:
        fn(f, os.path.getsize(dst))
    return dst


def _table(f):
    f.seek(68)
    n, toff = struct.unpack("<QQ", f.read(16))
    return n, toff


def _put(f, off, fmt, *v):
    f.seek(off)
    f.write(struct.pack(fmt, *v))


def _first_quant(f):
    n, toff = _table(f)
    for i in range(n):
        f.seek(toff + i * REC + 64)
        kind = struct.unpack("<I", f.read(4))[0]
        if kind == 1:
            return toff + i * REC
    raise AssertionError("no quantized record")


CASES = {
    "valid": (lambda f, sz: None, True),
    "truncated header": (lambda f, sz: f.truncate(1000), False),
    "bad magic": (lambda f, sz: _put(f, 0, "<4s", b"SSX "), False),
    "newer format version": (lambda f, sz: _put(f, 4, "<I", 10), False),
    "invalid level count": (lambda f, sz: _put(f, 48, "<I", 0), False),
    "unsupported flags": (lambda f, sz: _put(f, 152, "<I", 64), False),
    "minneg without scale6": (lambda f, sz: _put(f, 152, "<I", 4), False),
    "tensor table out of bounds": (lambda f, sz: _put(f, 76, "<Q", sz + 4096), False),
    "zero tensor dimensions": (lambda f, sz: _put(f, _first_quant(f) + 68, "<I", 0), False),
    "unknown tensor kind": (lambda f, sz: _put(f, _first_quant(f) + 64, "<I", 7), False),
    "invalid flat code width": (lambda f, sz: _put(f, _first_quant(f) + 244, "<I", 9), False),
    "quantized codes out of bounds": (lambda f, sz: _put(f, _first_quant(f) + 176, "<Q", sz - 8), False),
    "metadata out of bounds": (lambda f, sz: _put(f, _first_quant(f) + 96, "<Q", sz), False),
    "f32 payload size wrong": (lambda f, sz: _put(f, _f32_rec(f) + 88, "<Q", 12), False),
}


def _f32_rec(f):
    n, toff = _table(f)
    for i in range(n):
        f.seek(toff + i * REC + 64)
        if struct.unpack("<I", f.read(4))[0] == 0:
            return toff + i * REC
    raise AssertionError("no f32 record")


@pytest.mark.parametrize("case", sorted(CASES))
def test_loader_accepts_and_rejects(case):
    fn, valid = CASES[case]
    path = _mutate(fn)
    ok, why = sheep_b200.ssf_check(path)
    assert bool(ok) == valid, why
    if not valid:
        assert why
    if helpers.have_ref() and case not in ("minneg without scale6",):
        # the reference loader agrees (sml_model_open; a spawned process)
        import concurrent.futures as cf
        import multiprocessing as mp
        with cf.ProcessPoolExecutor(max_workers=1, mp_context=mp.get_context("spawn")) as ex:
            ref_ok = ex.submit(_ref_open, path).result()
        assert ref_ok == valid


def _ref_open(path):
    import ctypes
    L = helpers._ref_lib()
    h = L.refh_open(path.encode(), 64, 1, 0)
    if h:
        L.refh_close(ctypes.c_void_p(h))
    return bool(h)


def test_nccl_id_without_gpu():
    """The expert-parallel layer's NCCL id comes from the library with NCCL
    loaded at run time and no GPU needed; each call makes a new one."""
    import sheep_b200
    a, b = sheep_b200.nccl_unique_id(), sheep_b200.nccl_unique_id()
    assert len(a) == 128 and len(b) == 128 and a != b


def test_expert_ranges_cover_every_expert_once():
    from sheep_b200 import dist as sd
    for ne in (8, 16, 60, 128, 256):
        for world in (1, 2, 3, 4, 8):
            got = [e for r in range(world) for e in range(*sd.expert_range(ne, world, r))]
            assert got == list(range(ne))
