"""sheep_b200: a B200-native decode engine for SML's SSF models.

The product is libsheep_b200.so (C ABI, include/sml-gpu.h and
include/sheep_b200.h): CUDA kernels for sm_100a behind the reference's
sml_gpu_* entry points. This module is a thin ctypes mirror of that ABI for
Python callers, tests and the bench. It never computes anything itself, and it
fails loudly when the library is missing rather than falling back to the CPU.
"""
import ctypes
import os

import numpy as np

from .configs import CONFIGS, spec_for  # noqa: F401

_HERE = os.path.dirname(os.path.abspath(__file__))
# SHEEP_B200_LIB selects another build of the same ABI (the checked build).
LIB_PATH = os.environ.get("SHEEP_B200_LIB") or os.path.join(_HERE, "lib", "libsheep_b200.so")
_lib = None


class SsfSpec(ctypes.Structure):
    """ssfgen_spec (include/sheep_b200.h)."""
    _fields_ = [(n, ctypes.c_uint32) for n in
                "n_layer n_embd n_head n_head_kv head_dim n_ff n_vocab".split()] + \
               [("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float)] + \
               [(n, ctypes.c_uint32) for n in
                "tied qkv_bias qk_norm nbits emb_nbits scale6 minneg "
                "n_expert n_expert_used moe_flags expert_ff perm_mode".split()] + \
               [("seed", ctypes.c_uint64), ("sigma", ctypes.c_float), ("threads", ctypes.c_int),
                ("direct", ctypes.c_uint32)]


def lib():
    """The loaded engine library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m sheep_b200.build` "
                           "(there is no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    vp, cp, ip, fp = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float)
    sig = {
        "sml_gpu_open": (ip, [cp, ip, ip, ip, cp, ip]),
        "sml_gpu_prefill": (fp, [vp, ip, ip]),
        "sml_gpu_step": (fp, [ip, ip]),
        "sml_gpu_layers": (ip, [vp]),
        "sml_gpu_prompt_mode": (None, [ip]),
        "sml_gpu_decode_cpu": (ip, [ip]),
        "sml_gpu_set_middle": (None, [ip, vp]),
        "sml_gpu_engine": (vp, []),
        "sml_gpu_close": (None, []),
        "sb_open": (vp, [cp, ip, cp, ip]),
        "sb_open_tp": (vp, [cp, ip, ip, ip, cp, ip]),
        "sb_tp_handle": (ip, [vp, vp]),
        "sb_set_prompt_mode": (ip, [vp, ip]),
        "sb_kv_rows": (ip, [vp, ip, ip, vp, vp]),
        "sb_prompt_splits": (ip, [vp, vp]),
        "sb_tp_connect": (ip, [vp, vp, cp, ip]),
        "sb_close": (None, [vp]),
        "sb_info": (None, [vp, vp]),
        "sb_bytes_per_token": (ctypes.c_uint64, [vp]),
        "sb_step": (fp, [vp, ip, ip]),
        "sb_prefill": (fp, [vp, vp, ip, ip]),
        "sb_generate": (ip, [vp, vp, ip, ip, vp]),
        "sb_generate_timed": (ip, [vp, vp, ip, ip, ip, vp, fp]),
        "sb_device_logits": (vp, [vp]),
        "sb_launches_per_token": (ip, [vp]),
        "sb_time_kernel": (ip, [vp, ip, ip, fp, ctypes.POINTER(ctypes.c_double)]),
        "sb_trace": (ip, [vp, vp, ip]),
        "sb_last_error": (cp, []),
        "sb_tset_open": (vp, [cp, cp, ip]),
        "sb_tset_close": (None, [vp]),
        "sb_tset_shape": (ip, [vp, cp, vp, vp, vp]),
        "sb_tset_bytes": (ctypes.c_ulonglong, [vp, cp]),
        "sb_tset_gemv_dev": (ip, [vp, cp, vp, ip, vp, vp]),
        "sb_tset_gemv_host": (ip, [vp, cp, vp, ip, vp]),
        "sb_tset_time_gemv": (ip, [vp, cp, vp, ip, ip, fp]),
        "sb_tset_gemm_tc": (ip, [vp, cp, vp, ip, ip, vp, vp]),
        "sb_tset_gemm_tc_host": (ip, [vp, cp, vp, ip, ip, vp]),
        "sb_tset_time_gemm_tc": (ip, [vp, cp, vp, ip, ip, ip, fp]),
        "sb_tset_requant8_host": (ip, [vp, cp, vp, vp]),
        "sb_tset_matvec": (ip, [vp, cp, vp, vp, vp, vp, vp]),
        "sb_tset_matvec_permuted": (ip, [vp, cp, vp, vp, vp, vp, vp]),
        "sb_tset_dequant_rows": (ip, [vp, cp, vp, ip, vp]),
        "sb_quantize_act": (ip, [vp, vp, ip, vp, vp, vp, vp]),
        "ssfgen_write": (ip, [cp, vp, cp, ip]),
        "sb_ssf_check": (ip, [cp, cp, ip]),
        "sb_draw_experts": (None, [ctypes.c_uint64]),
        "sb_attn_decode": (ip, [vp, vp, vp, vp, vp, vp, vp, ctypes.c_float, ip, ip, ip, ip, ip, ctypes.c_float,
                                vp, vp]),
        "sb_attn_last_error": (cp, []),
        "sb_attn_decode_noalloc": (ip, [vp, vp, vp, vp, vp, vp, vp, ctypes.c_float, ip, ip, ip, ip, ip,
                                        ctypes.c_float, vp, vp]),
        "sb_attn_noalloc_last_error": (cp, []),
        "sb_moe_open": (vp, [cp, ip, ip, cp, ip]),
        "sb_moe_close": (None, [vp]),
        "sb_moe_info": (None, [vp, vp]),
        "sb_moe_forward": (ip, [vp, vp, ip, vp, vp]),
        "sb_moe_forward_host": (ip, [vp, vp, ip, vp, vp, vp, vp]),
        "sb_moe_time": (ip, [vp, vp, ip, ip, fp, vp]),
        "sb_moe_route": (ip, [vp, ip, ip, ip, ctypes.c_uint, vp, vp, vp]),
        "sb_moe_last_error": (cp, []),
        "sb_moe_set_tensor_cores": (ip, [vp, ip]),
        "sb_moe_set_exchange": (ip, [vp, ip]),
        "sb_moe_a2a_plan": (ip, [ip, ip, ip, ip, vp, vp, vp, vp, vp, vp]),
        "sb_moe_open_ep": (vp, [cp, ip, ip, ip, ip, vp, cp, ip]),
        "sb_nccl_unique_id": (ip, [vp]),
        "sb_tc_imma": (ip, [vp, vp, vp, ip, ip, ip, vp, vp]),
        "sb_tc_last_error": (cp, []),
        "sb_tc_trace": (ip, [vp, ip]),
        "sb_batch_open": (vp, [cp, ip, ip, cp, ip]),
        "sb_batch_close": (None, [vp]),
        "sb_batch_info": (None, [vp, vp]),
        "sb_forward_multi": (fp, [vp, vp, vp]),
        "sb_batch_generate": (ip, [vp, vp, ip, ip, ip, vp, fp]),
        "sb_batch_device_logits": (vp, [vp]),
        "sb_batch_last_error": (cp, []),
        "sb_batch_kv": (ip, [vp, ip, ip, ip, vp, vp]),
        "sb_batch_open_paged": (vp, [cp, ip, ip, ip, cp, ip]),
        "sb_seq_new": (ip, [vp]),
        "sb_seq_free": (ip, [vp, ip]),
        "sb_seq_truncate": (ip, [vp, ip, ip]),
        "sb_forward_seqs": (fp, [vp, vp, vp, vp, ip]),
        "sb_batch_pages": (None, [vp, vp]),
        "sb_seq_kv": (ip, [vp, ip, ip, ip, vp, vp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def write_model(path, **spec):
    """Write a seeded synthetic SSF model (ssfgen_write)."""
    s = SsfSpec()
    for k, v in spec.items():
        setattr(s, k, v)
    why = ctypes.create_string_buffer(512)
    if not lib().ssfgen_write(path.encode(), ctypes.byref(s), why, 512):
        raise RuntimeError(why.value.decode())
    return path


def draw_experts(seed):
    """Engines opened after this fill their MoE experts on the device from
    `seed` (files written with direct=2 leave those bytes out); 0 restores
    reading them from the file (sb_draw_experts)."""
    lib().sb_draw_experts(int(seed))


def ssf_check(path):
    """(1, "") if the loader accepts the file, else (0, why). No GPU needed."""
    why = ctypes.create_string_buffer(512)
    ok = lib().sb_ssf_check(path.encode(), why, 512)
    return ok, why.value.decode()


class Engine:
    """A model on the GPU with its KV cache (the handle form of sml-gpu.h)."""

    def __init__(self, path, n_ctx=256, tp=None):
        """tp=(world, rank, dist): this rank of a tensor-parallel engine over
        `world` GPUs (dist: an initialised torch.distributed, used once to pass
        the ranks' exchange handles around); every rank must construct it."""
        why = ctypes.create_string_buffer(512)
        if tp is None or tp[0] == 1:
            self.h = lib().sb_open(path.encode(), n_ctx, why, 512)
        else:
            world, rank, dist = tp
            self.h = lib().sb_open_tp(path.encode(), n_ctx, world, rank, why, 512)
        if not self.h:
            raise RuntimeError(f"sb_open: {why.value.decode()}")
        if tp is not None and tp[0] > 1:
            world, rank, dist = tp
            hb = ctypes.create_string_buffer(64)
            if not lib().sb_tp_handle(self.h, hb):
                raise RuntimeError(f"sb_tp_handle: {lib().sb_last_error().decode()}")
            allh = [None] * world
            dist.all_gather_object(allh, bytes(hb.raw))
            joined = ctypes.create_string_buffer(b"".join(allh), 64 * world)
            if not lib().sb_tp_connect(self.h, joined, why, 512):
                raise RuntimeError(f"sb_tp_connect: {why.value.decode()}")
        info = (ctypes.c_int * 16)()
        lib().sb_info(self.h, info)
        (self.n_layer, self.n_embd, self.n_head, self.n_head_kv, self.head_dim, self.n_ff,
         self.n_vocab, self.n_ctx, self.n_expert, self.n_expert_used) = info[:10]
        self.bytes_per_token = int(lib().sb_bytes_per_token(self.h))

    def step(self, tok, pos):
        p = lib().sb_step(self.h, int(tok), int(pos))
        if not p:
            raise RuntimeError(f"sb_step failed: {lib().sb_last_error().decode()}")
        return np.ctypeslib.as_array(p, shape=(self.n_vocab,)).copy()

    def prompt_mode(self, level):
        """sml_gpu_prompt_mode on this engine: 0/1 step the prompt, 2 reads it in
        tensor-core chunks (all but the last token). Returns the level set."""
        return lib().sb_set_prompt_mode(self.h, int(level))

    def kv_rows(self, layer, pos):
        """The cached key and value rows of (layer, pos), fp16 bit patterns."""
        kvd = self.n_head_kv * self.head_dim
        k, v = np.zeros(kvd, np.uint16), np.zeros(kvd, np.uint16)
        if not lib().sb_kv_rows(self.h, int(layer), int(pos), _p(k), _p(v)):
            raise RuntimeError("sb_kv_rows failed")
        return k, v

    def prompt_splits(self):
        out = (ctypes.c_int * 5)()
        if not lib().sb_prompt_splits(self.h, out):
            raise RuntimeError(f"no tensor-core prompt path: {lib().sb_last_error().decode()}")
        return list(out)

    def prefill(self, ids, pos0=0):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        p = lib().sb_prefill(self.h, _p(ids), int(pos0), len(ids))
        if not p:
            raise RuntimeError(f"sb_prefill failed: {lib().sb_last_error().decode()}")
        return np.ctypeslib.as_array(p, shape=(self.n_vocab,)).copy()

    def generate(self, prompt, ngen, timed=False, warmup=0):
        """Greedy ids; with timed=True also the CUDA-event ms of the loop after
        `warmup` untimed tokens (ngen ids = ngen - 1 timed replays)."""
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(ngen + (warmup if timed else 0), np.int32)
        ms = ctypes.c_float(0)
        if timed:
            ok = lib().sb_generate_timed(self.h, _p(prompt), len(prompt), warmup, ngen, _p(out), ctypes.byref(ms))
        else:
            ok = lib().sb_generate(self.h, _p(prompt), len(prompt), ngen, _p(out))
        if not ok:
            raise RuntimeError(f"sb_generate failed: {lib().sb_last_error().decode()}")
        return (out, ms.value) if timed else out

    @property
    def launches_per_token(self):
        return lib().sb_launches_per_token(self.h)

    KERNELS = {"qkv": 0, "attn": 1, "o": 2, "ffn": 3, "down": 4, "head": 5}

    def time_kernel(self, which, reps):
        """(avg ms per launch, weight bytes per launch) of one kernel class, each
        launch alone; leaves the decode state undefined."""
        ms, by = ctypes.c_float(0), ctypes.c_double(0)
        if not lib().sb_time_kernel(self.h, self.KERNELS[which], reps, ctypes.byref(ms), ctypes.byref(by)):
            raise RuntimeError(f"sb_time_kernel failed: {lib().sb_last_error().decode()}")
        return ms.value, by.value

    def close(self):
        if self.h:
            lib().sb_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TensorSet:
    """Every flat tensor of an SSF file on the GPU, for kernel-level calls."""

    def __init__(self, path):
        why = ctypes.create_string_buffer(512)
        self.h = lib().sb_tset_open(path.encode(), why, 512)
        if not self.h:
            raise RuntimeError(f"sb_tset_open: {why.value.decode()}")

    def shape(self, name):
        r, c, b = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        if not lib().sb_tset_shape(self.h, name.encode(), ctypes.byref(r), ctypes.byref(c), ctypes.byref(b)):
            raise KeyError(name)
        return r.value, c.value, b.value

    def nbytes(self, name):
        return int(lib().sb_tset_bytes(self.h, name.encode()))

    def matvec(self, name, x, permuted=False):
        """y = W x and the int8 activation the kernel staged; permuted=True takes
        x already in the tensor's column order (the down projection's staging)."""
        rows, cols, _ = self.shape(name)
        x = np.ascontiguousarray(x, dtype=np.float32)
        assert x.shape == (cols,)
        y = np.zeros(rows, np.float32)
        q = np.zeros(cols, np.int8)
        s = np.zeros(cols // 32, np.float32)
        sums = np.zeros(cols // 32, np.int32)
        fn = lib().sb_tset_matvec_permuted if permuted else lib().sb_tset_matvec
        if not fn(self.h, name.encode(), _p(x), _p(y), _p(q), _p(s), _p(sums)):
            raise RuntimeError(f"sb_tset_matvec failed: {lib().sb_last_error().decode()}")
        return y, q, s, sums

    def dequant_rows(self, name, rows):
        _, cols, _ = self.shape(name)
        rows = np.ascontiguousarray(rows, dtype=np.int32)
        out = np.zeros((len(rows), cols), np.float32)
        if not lib().sb_tset_dequant_rows(self.h, name.encode(), _p(rows), len(rows), _p(out)):
            raise RuntimeError("sb_tset_dequant_rows failed")
        return out

    def gemv(self, name, X):
        """Y [nb, rows] = W X[b] for host rows X [nb, cols] (batched for nb > 1)."""
        rows, cols, _ = self.shape(name)
        X = np.ascontiguousarray(np.atleast_2d(X), np.float32)
        assert X.shape[1] == cols
        Y = np.zeros((len(X), rows), np.float32)
        if not lib().sb_tset_gemv_host(self.h, name.encode(), _p(X), len(X), _p(Y)):
            raise RuntimeError("sb_tset_gemv_host failed")
        return Y

    def time_gemv(self, name, X, reps):
        """Mean device ms of one GEMV over the host rows X, L2 flushed before each run."""
        X = np.ascontiguousarray(np.atleast_2d(X), np.float32)
        ms = ctypes.c_float()
        if not lib().sb_tset_time_gemv(self.h, name.encode(), _p(X), len(X), reps, ctypes.byref(ms)):
            raise RuntimeError("sb_tset_time_gemv failed")
        return ms.value

    def gemm_tc(self, name, X, split=1):
        """Y [nb, rows]: the batched path on the tensor cores (int8 per-256
        arithmetic); split > 1 sums that many runs of superblocks in run order."""
        rows, cols, _ = self.shape(name)
        X = np.ascontiguousarray(np.atleast_2d(X), np.float32)
        Y = np.zeros((len(X), rows), np.float32)
        if not lib().sb_tset_gemm_tc_host(self.h, name.encode(), _p(X), len(X), split, _p(Y)):
            raise RuntimeError("sb_tset_gemm_tc_host failed")
        return Y

    def time_gemm_tc(self, name, X, reps, split=1):
        X = np.ascontiguousarray(np.atleast_2d(X), np.float32)
        ms = ctypes.c_float()
        if not lib().sb_tset_time_gemm_tc(self.h, name.encode(), _p(X), len(X), split, reps, ctypes.byref(ms)):
            raise RuntimeError("sb_tset_time_gemm_tc failed")
        return ms.value

    def requant8(self, name):
        """(w8 [rows, nsb*256] int8, s8 [rows, nsb] float32) of the tensor-core path."""
        rows, cols, _ = self.shape(name)
        nsb = (cols // 32 + 7) // 8
        w8 = np.zeros((rows, nsb * 256), np.int8)
        s8 = np.zeros((rows, nsb), np.float32)
        if not lib().sb_tset_requant8_host(self.h, name.encode(), _p(w8), _p(s8)):
            raise RuntimeError("sb_tset_requant8_host failed")
        return w8, s8

    def gemv_dev(self, name, x_ptr, nb, y_ptr, stream=0):
        if not lib().sb_tset_gemv_dev(self.h, name.encode(), x_ptr, nb, y_ptr, stream):
            raise RuntimeError("sb_tset_gemv_dev failed")

    def close(self):
        if self.h:
            lib().sb_tset_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def nccl_unique_id():
    """128 bytes for sb_moe_open_ep, made by one process and shared by the host."""
    buf = ctypes.create_string_buffer(128)
    if not lib().sb_nccl_unique_id(buf):
        raise RuntimeError(f"sb_nccl_unique_id: {lib().sb_moe_last_error().decode()}")
    return buf.raw


class MoeLayer:
    """One mixture-of-experts FFN layer of an SSF file on the GPU (sb_moe_*).
    With ep=(world, rank, nccl_id) the experts are spread over `world` GPUs
    (one process each, every process passing all tokens)."""

    def __init__(self, path, layer=0, max_tokens=256, ep=None):
        why = ctypes.create_string_buffer(512)
        if ep is None:
            self.h = lib().sb_moe_open(path.encode(), layer, max_tokens, why, 512)
        else:
            world, rank, nid = ep
            idbuf = ctypes.create_string_buffer(bytes(nid), 128)
            self.h = lib().sb_moe_open_ep(path.encode(), layer, max_tokens, world, rank, idbuf, why, 512)
        if not self.h:
            raise RuntimeError(f"sb_moe_open: {why.value.decode()}")
        info = (ctypes.c_int * 16)()
        lib().sb_moe_info(self.h, info)
        self.n_embd, self.n_ff, self.n_expert, self.k, self.flags, self.max_tokens, self.nbits = info[:7]
        self.expert_bytes = (info[7] & 0xffffffff) | (info[8] << 32)
        self.router_bytes = info[9]
        self.world, self.rank, self.e_lo, self.e_hi = info[10:14]

    def forward(self, x):
        """y [T, n_embd], sel and w [T, k], distinct experts, from rows x [T, n_embd]."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        T = len(x)
        y = np.zeros_like(x)
        sel = np.zeros((T, self.k), np.int32)
        w = np.zeros((T, self.k), np.float32)
        na = ctypes.c_int()
        if not lib().sb_moe_forward_host(self.h, _p(x), T, _p(y), _p(sel), _p(w), ctypes.byref(na)):
            raise RuntimeError(f"sb_moe_forward_host: {lib().sb_moe_last_error().decode()}")
        return y, sel, w, na.value

    def exchange(self, mode):
        """An expert-parallel handle's exchange: "all-reduce" (every rank passes
        all tokens) or "all-to-all" (every rank passes its own tokens)."""
        if not lib().sb_moe_set_exchange(self.h, {"all-reduce": 0, "all-to-all": 1}[mode]):
            raise RuntimeError(f"sb_moe_set_exchange: {lib().sb_moe_last_error().decode()}")

    def tensor_cores(self, on):
        """Calls of 16+ rows on the tensor cores (True), on the integer kernels
        (False), or "auto" (the default: the tensor cores from 8 chosen rows
        per expert on average); returns whether this handle can use the tensor
        cores."""
        return bool(lib().sb_moe_set_tensor_cores(self.h, 2 if on == "auto" else 1 if on else 0))

    def forward_dev(self, x_ptr, n_tok, y_ptr, stream=0):
        if not lib().sb_moe_forward(self.h, x_ptr, n_tok, y_ptr, stream):
            raise RuntimeError(f"sb_moe_forward: {lib().sb_moe_last_error().decode()}")

    def time(self, x, reps):
        """(mean device ms of one forward with L2 flushed before each, distinct experts)."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        ms, na = ctypes.c_float(), ctypes.c_int()
        if not lib().sb_moe_time(self.h, _p(x), len(x), reps, ctypes.byref(ms), ctypes.byref(na)):
            raise RuntimeError(f"sb_moe_time: {lib().sb_moe_last_error().decode()}")
        return ms.value, na.value

    def close(self):
        if self.h:
            lib().sb_moe_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Batch:
    """n_seq conversations decoding together on the GPU (sb_batch_*): the
    reference's sml_forward_multi with every product on the tensor cores."""

    def __init__(self, path, n_seq, n_ctx):
        why = ctypes.create_string_buffer(512)
        self.h = lib().sb_batch_open(path.encode(), n_seq, n_ctx, why, 512)
        if not self.h:
            raise RuntimeError(f"sb_batch_open: {why.value.decode()}")
        info = (ctypes.c_int * 16)()
        lib().sb_batch_info(self.h, info)
        self.n_seq, self.n_ctx, self.n_vocab = info[0], info[1], info[2]
        self.splits = list(info[3:8])
        self.file_bytes = (info[8] & 0xffffffff) | (info[9] << 32)
        self.int8_bytes = (info[10] & 0xffffffff) | (info[11] << 32)
        self.launches = info[12]
        self.tile_tokens = info[13]
        self.expert_bytes = (info[14] & 0xffffffff) | (info[15] << 32)

    def forward_multi(self, tokens, pos):
        """logits [n_seq, n_vocab] for tokens[s] at pos[s] (pos < 0: idle slot)."""
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(pos, np.int32)
        assert len(t) == self.n_seq and len(p) == self.n_seq
        r = lib().sb_forward_multi(self.h, _p(t), _p(p))
        if not r:
            raise RuntimeError(f"sb_forward_multi: {lib().sb_batch_last_error().decode()}")
        return np.ctypeslib.as_array(r, shape=(self.n_seq * self.n_vocab,)).reshape(self.n_seq, self.n_vocab).copy()

    def generate(self, prompts, ngen, nwarm=0, timed=False):
        """ids [n_seq, nwarm + ngen] greedy from prompts [n_seq, np] (and the
        device ms of the last ngen - 1 steps when timed)."""
        P = np.ascontiguousarray(prompts, np.int32)
        ids = np.zeros((self.n_seq, nwarm + ngen), np.int32)
        ms = ctypes.c_float()
        if not lib().sb_batch_generate(self.h, _p(P), P.shape[1], nwarm, ngen, _p(ids),
                                       ctypes.byref(ms) if timed else None):
            raise RuntimeError(f"sb_batch_generate: {lib().sb_batch_last_error().decode()}")
        return (ids, ms.value) if timed else ids

    def kv(self, layer, slot, pos, n_kv_dim):
        """(k, v) cached fp16 rows (as uint16) of slot at pos in layer."""
        k = np.zeros(n_kv_dim, np.uint16)
        v = np.zeros(n_kv_dim, np.uint16)
        if not lib().sb_batch_kv(self.h, layer, slot, pos, _p(k), _p(v)):
            raise RuntimeError(f"sb_batch_kv: {lib().sb_batch_last_error().decode()}")
        return k, v

    def close(self):
        if self.h:
            lib().sb_batch_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


class PagedBatch:
    """Continuous batching over a paged KV cache (sb_batch_open_paged): up to
    n_slots live sequences per step, in any slots, each holding pages of 64
    positions from a pool of n_pages."""

    def __init__(self, path, n_slots, n_ctx, n_pages):
        why = ctypes.create_string_buffer(512)
        self.h = lib().sb_batch_open_paged(path.encode(), n_slots, n_ctx, n_pages, why, 512)
        if not self.h:
            raise RuntimeError(f"sb_batch_open_paged: {why.value.decode()}")
        info = (ctypes.c_int * 16)()
        lib().sb_batch_info(self.h, info)
        self.n_slots, self.n_ctx, self.n_vocab = info[0], info[1], info[2]

    def new_seq(self):
        s = lib().sb_seq_new(self.h)
        if s < 0:
            raise RuntimeError(f"sb_seq_new: {lib().sb_batch_last_error().decode()}")
        return s

    def free_seq(self, seq):
        if not lib().sb_seq_free(self.h, seq):
            raise RuntimeError(f"sb_seq_free: {lib().sb_batch_last_error().decode()}")

    def truncate(self, seq, n):
        if not lib().sb_seq_truncate(self.h, seq, n):
            raise RuntimeError(f"sb_seq_truncate: {lib().sb_batch_last_error().decode()}")

    def forward(self, seqs, tokens, pos):
        """logits [len(seqs), n_vocab]: slot s runs sequence seqs[s] with tokens[s] at pos[s]."""
        q = np.ascontiguousarray(seqs, np.int32)
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(pos, np.int32)
        assert len(q) == len(t) == len(p)
        r = lib().sb_forward_seqs(self.h, _p(q), _p(t), _p(p), len(q))
        if not r:
            raise RuntimeError(f"sb_forward_seqs: {lib().sb_batch_last_error().decode()}")
        return np.ctypeslib.as_array(r, shape=(len(q) * self.n_vocab,)).reshape(len(q), self.n_vocab).copy()

    def pages(self):
        """(pages in the pool, free pages, live sequences)."""
        out = (ctypes.c_int * 4)()
        lib().sb_batch_pages(self.h, out)
        return out[0], out[1], out[2]

    def kv(self, layer, seq, pos, n_kv_dim):
        k = np.zeros(n_kv_dim, np.uint16)
        v = np.zeros(n_kv_dim, np.uint16)
        if not lib().sb_seq_kv(self.h, layer, seq, pos, _p(k), _p(v)):
            raise RuntimeError("sb_seq_kv failed")
        return k, v

    def close(self):
        if self.h:
            lib().sb_batch_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def moe_a2a_plan(world, rank, n_expert, sels):
    """The all-to-all exchange's plan of `rank` (sb_moe_a2a_plan, host only):
    sels[r] is rank r's [n_tok, k] chosen experts. Returns (send_cnt,
    recv_cnt, send_slot, recv_expert, chunks)."""
    k = sels[0].shape[1]
    n_tok = np.array([len(s_) for s_ in sels], np.int32)
    sel = np.ascontiguousarray(np.concatenate([np.asarray(s_, np.int32).reshape(-1) for s_ in sels]), np.int32)
    send_cnt, recv_cnt = np.zeros(world, np.int32), np.zeros(world, np.int32)
    send_slot = np.zeros(max(1, n_tok[rank] * k), np.int32)
    recv_exp = np.zeros(max(1, len(sel)), np.int32)
    nch = lib().sb_moe_a2a_plan(world, rank, n_expert, k, _p(n_tok), _p(sel), _p(send_cnt), _p(recv_cnt),
                                _p(send_slot), _p(recv_exp))
    if nch < 0:
        raise RuntimeError("sb_moe_a2a_plan: bad input")
    return send_cnt, recv_cnt, send_slot[:int(send_cnt.sum())], recv_exp[:int(recv_cnt.sum())], nch


def moe_route_dev(logits_ptr, n_tok, n_expert, k, flags, sel_ptr, w_ptr, stream=0):
    """Routing alone on device buffers (sb_moe_route)."""
    if not lib().sb_moe_route(logits_ptr, n_tok, n_expert, k, flags, sel_ptr, w_ptr, stream):
        raise RuntimeError(f"sb_moe_route: {lib().sb_moe_last_error().decode()}")


# ----------------------------------------------------------------- sml-gpu.h mirror
# Same names, argument meaning and error behaviour as the reference's C API
# (sml/sml-gpu.h:11-34), for Python callers.

def sml_gpu_open(path, n_ctx=0, threads=0, gpu_layers=0):
    """Returns (1, "") or (0, why)."""
    why = ctypes.create_string_buffer(512)
    ok = lib().sml_gpu_open(path.encode(), n_ctx, threads, gpu_layers, why, 512)
    return ok, why.value.decode()


def _n_vocab():
    info = (ctypes.c_int * 16)()
    lib().sb_info(lib().sml_gpu_engine(), info)
    return info[6]


def sml_gpu_prefill(ids, pos0, n=None):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    p = lib().sml_gpu_prefill(_p(ids), pos0, len(ids) if n is None else n)
    return None if not p else np.ctypeslib.as_array(p, shape=(_n_vocab(),)).copy()


def sml_gpu_step(tok, pos, copy=True):
    """Host logits of `tok` at `pos`. copy=False returns a view of the library's
    own buffer, as a C caller sees it: valid until the next call."""
    p = lib().sml_gpu_step(tok, pos)
    if not p:
        return None
    a = np.ctypeslib.as_array(p, shape=(_n_vocab(),))
    return a.copy() if copy else a


def sml_gpu_layers():
    of = ctypes.c_int()
    n = lib().sml_gpu_layers(ctypes.byref(of))
    return n, of.value


def sml_gpu_prompt_mode(level):
    lib().sml_gpu_prompt_mode(level)


def sml_gpu_decode_cpu(on):
    return lib().sml_gpu_decode_cpu(on)


def sml_gpu_set_middle(layers, fn=None):
    lib().sml_gpu_set_middle(layers, None)


def sml_gpu_close():
    lib().sml_gpu_close()
