"""Test helpers: synthetic models, the CPU checkers, the reference build.

The checkers are test infrastructure: oracle/_build/liboracle.so (this
repository's C restatement) and oracle/_ref/libsmlref.so (the reference's own
CPU code, when it was built). Neither is ever used by the engine.

The reference keeps its group-field width as process-global state
(sml/sml-model.c:225-250), so every call into it runs in a fresh spawned
process.
"""
import concurrent.futures as cf
import ctypes
import hashlib
import json
import multiprocessing as mp
import os
import subprocess
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
ORACLE_LIB = os.path.join(ORACLE_DIR, "_build", "liboracle.so")
REF_LIB = os.path.join(ORACLE_DIR, "_ref", "libsmlref.so")
MODEL_DIR = os.path.join(tempfile.gettempdir(), "sheep_b200_models")


def build_oracle():
    subprocess.run(["make", "-s", "-C", ORACLE_DIR, "oracle"], check=True)
    ref = os.environ.get("SML_REFERENCE")
    if ref:
        subprocess.run(["make", "-s", "-C", ORACLE_DIR, "ref", "REF=" + ref], check=True)


def have_ref():
    return os.path.exists(REF_LIB)


def model_path(spec):
    """A synthetic SSF for `spec` (cached by its content)."""
    import sheep_b200
    os.makedirs(MODEL_DIR, exist_ok=True)
    key = hashlib.sha1(json.dumps(spec, sort_keys=True).encode()).hexdigest()[:16]
    path = os.path.join(MODEL_DIR, key + ".ssf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        sheep_b200.write_model(tmp, **spec)
        os.replace(tmp, path)
    return path


# The letters a-z are the vocabulary's only byte tokens (ids 0..25): a prompt
# of lowercase letters encodes one id per letter. Every other id but the last is
# a filler spelled "[id]", the last is the end-of-text special.
VOCAB_LETTERS = "abcdefghijklmnopqrstuvwxyz"


def with_vocab(path):
    """A copy of the SSF at `path` with a binary vocabulary appended (the
    layout sml_vocab_init reads, sml/sml-vocab.c:64-79: n_tokens, n_merges,
    bos, eos, offsets[n_tokens + 1], the token bytes, no merges) and the
    header's tok_off / tok_n pointing at it. Token strings are in the GPT-2
    byte-to-symbol spelling the reference's encoder looks up; letters and the
    characters of "[0123456789]" spell themselves in it."""
    import struct
    out = path[:-4] + ".vocab.ssf"
    if os.path.exists(out):
        return out
    with open(path, "rb") as f:
        data = bytearray(f.read())
    nv = struct.unpack_from("<I", data, 28)[0]
    toks = [c.encode() for c in VOCAB_LETTERS]
    toks += [f"[{i}]".encode() for i in range(len(toks), nv - 1)]
    toks.append(b"<|endoftext|>")
    offs, pos = [], 0
    for t in toks:
        offs.append(pos)
        pos += len(t)
    offs.append(pos)
    blob = struct.pack("<4I", nv, 0, nv - 1, nv - 1) + struct.pack(f"<{nv + 1}I", *offs) + b"".join(toks)
    tok_off = (len(data) + 15) // 16 * 16
    data += b"\0" * (tok_off - len(data)) + blob
    struct.pack_into("<2Q", data, 100, tok_off, len(blob))   # ssf header: tok_off, tok_n
    tmp = out + f".tmp{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(data)
    os.replace(tmp, out)
    return out


def vocab_ids(text):
    """Token ids of a reply written with with_vocab's vocabulary."""
    import re
    ids = []
    for m in re.finditer(r"\[(\d+)\]|([a-z])", text):
        ids.append(int(m.group(1)) if m.group(1) else VOCAB_LETTERS.index(m.group(2)))
    return ids


def file_sha(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(1 << 22), b""):
            h.update(b)
    return h.hexdigest()


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


# ------------------------------------------------------------------ restatement

class Oracle:
    """ctypes view of oracle/_build/liboracle.so (one model)."""

    _L = None

    @classmethod
    def lib(cls):
        if cls._L is None:
            L = ctypes.CDLL(ORACLE_LIB)
            L.so_open.restype = ctypes.c_void_p
            L.so_open.argtypes = [ctypes.c_char_p, ctypes.c_int]
            for n in ("so_close",):
                getattr(L, n).argtypes = [ctypes.c_void_p]
            cls._L = L
        return cls._L

    def __init__(self, path, n_ctx=256):
        self.m = ctypes.c_void_p(self.lib().so_open(path.encode(), n_ctx))
        assert self.m.value, path
        info = (ctypes.c_int * 8)()
        self.lib().so_info(self.m, info)
        self.info = list(info)
        self.n_vocab = info[6]

    def matvec(self, name, x, rows):
        y = np.zeros(rows, np.float32)
        assert self.lib().so_matvec(self.m, name.encode(), _p(np.ascontiguousarray(x, np.float32)), _p(y), 0, rows)
        return y

    def dequant_row(self, name, row, cols):
        out = np.zeros(cols, np.float32)
        assert self.lib().so_dequant_row(self.m, name.encode(), row, _p(out))
        return out

    def codes_row(self, name, row, cols):
        out = np.zeros(cols, np.uint8)
        assert self.lib().so_codes_row(self.m, name.encode(), row, _p(out))
        return out

    def forward(self, tok, pos):
        lg = np.zeros(self.n_vocab, np.float32)
        self.lib().so_forward(self.m, tok, pos, _p(lg))
        return lg

    def decode(self, prompt, ngen):
        prompt = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(ngen, np.int32)
        lg = np.zeros((ngen, self.n_vocab), np.float32)
        self.lib().so_decode(self.m, _p(prompt), len(prompt), ngen, _p(ids), _p(lg))
        return ids, lg

    def moe_ffn(self, layer, x, kmax=16):
        """The MoE FFN of `layer` on normalized rows x [T, E]: y [T, E], sel and w [T, k]."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        y = np.zeros_like(x)
        sel = np.zeros((len(x), kmax), np.int32)
        w = np.zeros((len(x), kmax), np.float32)
        k = 0
        for t in range(len(x)):
            k = self.lib().so_moe_ffn(self.m, layer, _p(x[t]), _p(y[t]), _p(sel[t]), _p(w[t]))
            assert k > 0, "layer has no router"
        return y, sel[:, :k], w[:, :k]

    def moe_expert(self, layer, e, x):
        """One expert's unweighted FFN output on a normalized row."""
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros_like(x)
        assert self.lib().so_moe_expert(self.m, layer, e, _p(x), _p(y))
        return y

    def requant8(self, name, rows, cols):
        nsb = (cols // 32 + 7) // 8
        w8 = np.zeros((rows, nsb * 256), np.int8)
        s8 = np.zeros((rows, nsb), np.float32)
        assert self.lib().so_requant8(self.m, name.encode(), _p(w8), _p(s8))
        return w8, s8

    def gemm_sb(self, name, X, rows):
        X = np.ascontiguousarray(np.atleast_2d(X), np.float32)
        Y = np.zeros((len(X), rows), np.float32)
        assert self.lib().so_gemm_sb(self.m, name.encode(), _p(X), len(X), _p(Y))
        return Y

    def gemm_sb_split(self, name, X, rows, split):
        X = np.ascontiguousarray(np.atleast_2d(X), np.float32)
        Y = np.zeros((len(X), rows), np.float32)
        assert self.lib().so_gemm_sb_split(self.m, name.encode(), _p(X), len(X), split, _p(Y))
        return Y

    def close(self):
        if self.m:
            self.lib().so_close(self.m)
            self.m = None


class OracleBatch:
    """so_batch_*: ns sequences with their own caches; mode 0 the decode
    arithmetic, mode 1 the batched (tensor-core) arithmetic."""

    def __init__(self, orc, ns, mode, splits=None):
        L = Oracle.lib()
        L.so_batch_open.restype = ctypes.c_void_p
        L.so_batch_open.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.so_batch_step.argtypes = [ctypes.c_void_p] * 4
        L.so_batch_set_splits.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.so_batch_close.argtypes = [ctypes.c_void_p]
        self.orc, self.ns = orc, ns
        self.b = ctypes.c_void_p(L.so_batch_open(orc.m, ns, mode))
        if splits is not None:
            sp = np.ascontiguousarray(splits, np.int32)
            L.so_batch_set_splits(self.b, _p(sp))

    def step(self, tokens, pos):
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(pos, np.int32)
        lg = np.zeros((self.ns, self.orc.n_vocab), np.float32)
        assert Oracle.lib().so_batch_step(self.b, _p(t), _p(p), _p(lg))
        return lg

    def kv(self, layer, slot, pos, n_kv_dim):
        k = np.zeros(n_kv_dim, np.uint16)
        v = np.zeros(n_kv_dim, np.uint16)
        L = Oracle.lib()
        L.so_batch_kv.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                  ctypes.c_void_p]
        assert L.so_batch_kv(self.b, layer, slot, pos, _p(k), _p(v))
        return k, v

    def close(self):
        if self.b:
            Oracle.lib().so_batch_close(self.b)
            self.b = None


def oracle_quant(x):
    x = np.ascontiguousarray(x, np.float32)
    n = len(x)
    q = np.zeros(n, np.int8)
    s = np.zeros(n // 32, np.float32)
    sums = np.zeros(n // 32, np.int32)
    Oracle.lib().so_quantize_act(_p(x), n, _p(q), _p(s), _p(sums))
    return q, s, sums


def oracle_quant_sb(x):
    x = np.ascontiguousarray(x, np.float32)
    n = len(x)
    q = np.zeros(n, np.int8)
    s = np.zeros(n // 32, np.float32)
    sums = np.zeros(n // 32, np.int32)
    Oracle.lib().so_quantize_act_sb(_p(x), n, _p(q), _p(s), _p(sums))
    return q, s, sums


def oracle_route(lg, k, flags=1):
    lg = np.ascontiguousarray(lg, np.float32)
    sel = np.zeros(16, np.int32)
    w = np.zeros(16, np.float32)
    got = Oracle.lib().so_moe_route(_p(lg), len(lg), k, flags, _p(sel), _p(w))
    return sel[:got], w[:got]


# ------------------------------------------------------------------ reference

def _ref_lib():
    L = ctypes.CDLL(REF_LIB)
    L.refh_open.restype = ctypes.c_void_p
    L.refh_open.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.refh_bytes_per_token.restype = ctypes.c_ulonglong
    return L


def _ref_task(kind, path, args):
    L = _ref_lib()
    if kind in ("quant", "quant_sb"):
        x = np.ascontiguousarray(args["x"], np.float32)
        n = len(x)
        q, s, sums = np.zeros(n, np.int8), np.zeros(n // 32, np.float32), np.zeros(n // 32, np.int32)
        (L.refh_quantize_act if kind == "quant" else L.refh_quantize_act_sb)(_p(x), n, _p(q), _p(s), _p(sums))
        return q, s, sums
    if kind == "multi":
        # sml_forward_multi over ns conversations, each its own context; steps
        # of (tokens, positions), a position < 0 leaving that slot out of the
        # call. env: SML_MULTI etc. as the reference reads them.
        for k, v in args.get("env", {}).items():
            os.environ[k] = v
        ns, nv = args["ns"], args["n_vocab"]
        L.refh_forward_multi.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_void_p]
        hs = [L.refh_open(path.encode(), args.get("n_ctx", 64), args.get("threads", 4), 1) for _ in range(ns)]
        outs = []
        try:
            for tok, pos in args["steps"]:
                idx = [i for i in range(ns) if pos[i] >= 0]
                lg = np.zeros((len(idx), nv), np.float32)
                sub = (ctypes.c_void_p * len(idx))(*[hs[i] for i in idx])
                tk = np.ascontiguousarray([tok[i] for i in idx], np.int32)
                ps = np.ascontiguousarray([pos[i] for i in idx], np.int32)
                L.refh_forward_multi(sub, _p(tk), _p(ps), len(idx), _p(lg))
                full = np.zeros((ns, nv), np.float32)
                full[idx] = lg
                outs.append(full)
        finally:
            for h in hs:
                L.refh_close(ctypes.c_void_p(h))
        return np.array(outs)
    if kind == "route":
        lg = np.ascontiguousarray(args["lg"], np.float32)
        sel, w = np.zeros(16, np.int32), np.zeros(16, np.float32)
        got = L.refh_moe_route(_p(lg), len(lg), args["k"], args.get("flags", 1), ctypes.c_float(0.0), _p(sel), _p(w))
        return sel[:got], w[:got]
    with_ctx = 1 if kind in ("decode", "forward") else 0
    h = ctypes.c_void_p(L.refh_open(path.encode(), args.get("n_ctx", 256), args.get("threads", 4), with_ctx))
    if not h.value:
        raise RuntimeError(f"reference could not open {path}")
    try:
        if kind == "matvec":
            x = np.ascontiguousarray(args["x"], np.float32)
            rows, cols = args["rows"], len(x)
            y = np.zeros(rows, np.float32)
            q, s, sums = np.zeros(cols, np.int8), np.zeros(cols // 32, np.float32), np.zeros(cols // 32, np.int32)
            assert L.refh_matvec(h, args["name"].encode(), _p(x), _p(y), 0, rows, _p(q), _p(s), _p(sums))
            return y, q, s, sums
        if kind == "dequant":
            out = np.zeros((len(args["rows"]), args["cols"]), np.float32)
            for i, r in enumerate(args["rows"]):
                assert L.refh_dequant_row(h, args["name"].encode(), int(r), _p(out[i]))
            return out
        if kind == "decode":
            info = (ctypes.c_int * 8)()
            nv = L.refh_info(h, info)
            prompt = np.ascontiguousarray(args["prompt"], np.int32)
            ngen = args["ngen"]
            ids = np.zeros(ngen, np.int32)
            lg = np.zeros((ngen, nv), np.float32)
            assert L.refh_decode(h, _p(prompt), len(prompt), ngen, _p(ids), _p(lg))
            return ids, lg
        if kind == "forward":   # teacher-forced: logits after every token of `tokens`
            info = (ctypes.c_int * 8)()
            nv = L.refh_info(h, info)
            toks = args["tokens"]
            lg = np.zeros((len(toks), nv), np.float32)
            for i, t in enumerate(toks):
                L.refh_forward(h, int(t), i, _p(lg[i]))
            return lg
        if kind == "bytes":
            return int(L.refh_bytes_per_token(h))
    finally:
        L.refh_close(h)
    raise ValueError(kind)


def ref(kind, path=None, **args):
    """Run one reference call in a fresh spawned process."""
    with cf.ProcessPoolExecutor(max_workers=1, mp_context=mp.get_context("spawn")) as ex:
        return ex.submit(_ref_task, kind, path, args).result()


def rel_rms(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.sqrt(np.mean((a - b) ** 2)) / (np.sqrt(np.mean(a ** 2)) + 1e-30))


def agree_with_ties(ref_logits, got_logits):
    """Top-1 agreement under the reference's tie rule (sml/sml-gpu-fwd.c:2586-2598):
    a different top-1 is a tie when the reference's own logits for the two
    tokens are within 1% of its logits' standard deviation."""
    ac, ag = int(np.argmax(ref_logits)), int(np.argmax(got_logits))
    if ac == ag:
        return True, False
    sd = float(np.std(ref_logits.astype(np.float64)))
    tie = float(ref_logits[ac]) - float(ref_logits[ag]) <= 0.01 * sd
    return tie, tie


# ------------------------------------------------------------------ file reading

REC_FMT = "<64s4I2Q2Q2Q2Q2Q2Q4Q4Q2I"   # the 248-byte SSF record


def read_records(path):
    """name -> dict of the record's fields (tooling/sml_format.py:76-88 REC_FMT)."""
    import struct
    with open(path, "rb") as f:
        head = f.read(4096)
        n_tensors, table_off = struct.unpack_from("<QQ", head, 68)
        f.seek(table_off)
        raw = f.read(n_tensors * 248)
    out = {}
    names = ("kind rows cols group off nbytes sd_off sd_n sq_off sq_n perm_off perm_n "
             "md_off md_n mq_off mq_n c0 c1 c2 c3 n0 n1 n2 n3 layout nbits").split()
    for i in range(n_tensors):
        v = struct.unpack_from(REC_FMT, raw, i * 248)
        out[v[0].rstrip(b"\0").decode()] = dict(zip(names, v[1:]))
    return out


def read_perm(path, name):
    r = read_records(path)[name]
    return np.fromfile(path, dtype=np.int32, count=r["cols"], offset=r["perm_off"])
