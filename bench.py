"""Benchmark: greedy decode of the Qwen2.5-1.5B-shaped Q4 model at batch 1.

One step = one decode token (one pass of the decode path over one token).
The model is the seeded synthetic SSF of configuration 0 (28 layers, hidden
1536, 12/2 heads x 128, SwiGLU 8960, vocab 151936 tied, Q4 with 8-bit group
fields, q/k/v biases). Weights are 0.89 GB per token, far above the 126 MB L2,
so nothing is flushed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl sheep|reference]

value: device-resident greedy loop (one CUDA-graph replay per token, the
token chosen on the GPU), CUDA events over K tokens after a 128-token prompt
and W warm-up tokens. With N GPUs the one stream is split over them (tensor
parallelism: attention replicated, gate/up, down and head rows split, rows
exchanged over NVLink by the GEMVs), the max over ranks; strong scaling.
e2e: the same tokens through the reference-facing C ABI (sml_gpu_prefill /
sml_gpu_step with host ids in and host logits out, host argmax), wall clock.
--impl reference: the reference engine's own CPU decode (oracle/_ref, built
from its unchanged sources) on the box's host cores, same model and metric.
extras (single GPU only): configuration 1's GEMV microbench (GB/s of weight
bytes streamed, Q4 and Q8, batch 1/4/16) and configuration 2's MoE layer
(Qwen3-30B-A3B shape at 1/16/64/256 tokens a step: tok/s and GB/s of the
experts actually read plus the router), each run timed alone by CUDA events
with a 512 MB buffer rewritten before it, so the weights come from HBM; and
configuration 3's batch-1 decode (Llama-3-8B shape, 4.2 GB per token) and its
batched serving at 64 slots (2048-id prompts, 256 generated ids each).
extras with N > 1 GPUs: configuration 3 split the same way over the N GPUs,
configuration 2's MoE layer spread over them (expert parallelism,
sb_moe_open_ep, with the all-reduce and the all-to-all exchanges), the max
over ranks at 1/16/64/256 tokens, and configuration 4's batch-1 decode with
each layer's experts spread over the GPUs.
"""
import argparse
import ctypes
import json
import os
import re
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (batch 1 & 64, Q4); GEMV/MoE achieved HBM GB/s vs ~8 TB/s peak"
WORKLOAD = "qwen2.5-1.5b-shape Q4 greedy decode, batch 1, 128-token prompt"
PROMPT_LEN = 128
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libsmlref.so")


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(name):
    """Bytes per launch of a kernel from its committed ncu summary
    (profiles/<name>.md, a line `traffic_bytes_per_launch: N`), else None."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    try:
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", open(path).read())
        return int(m.group(1)) if m else None
    except OSError:
        return None


def model_path(spec, rank, dist, own_process=False):
    """The synthetic SSF of `spec` (written once, cached by content). With
    own_process the writer runs in a separate Python process, so the caller
    (the reference arm) never maps this repository's engine library."""
    d = os.path.join(tempfile.gettempdir(), "sheep_b200_bench")
    os.makedirs(d, exist_ok=True)
    import hashlib
    key = hashlib.sha1(json.dumps(spec, sort_keys=True).encode()).hexdigest()[:16]
    path = os.path.join(d, key + ".ssf")
    if rank == 0 and not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        if own_process:
            code = ("import json, sys; sys.path.insert(0, %r); import sheep_b200; "
                    "sheep_b200.write_model(%r, **json.loads(%r))" % (ROOT, tmp, json.dumps(spec)))
            subprocess.run([sys.executable, "-c", code], check=True)
        else:
            import sheep_b200
            sheep_b200.write_model(tmp, **spec)
        os.replace(tmp, path)
    if dist is not None:
        dist.barrier()
    return path


def bench_config(W, K):
    """The workload, identical in both arms."""
    return {"workload": WORKLOAD, "quant": "SSF v8 flat Q4", "batch": 1, "prompt": PROMPT_LEN,
            "seq_len": PROMPT_LEN + W + K}


class Clocks:
    """nvidia-smi clock and throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.path = tempfile.mktemp(suffix=".csv")
        self.proc = None

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        try:
            rows = [l.split(",") for l in open(self.path).read().strip().splitlines()]
        except OSError:
            rows = []
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_decode(path, n_prompt, nwarm, ngen, threads):
    """Reference CPU decode (oracle/_ref): prompt stepped, then greedy tokens;
    returns (tok/s over the timed ngen tokens, seconds, the greedy ids after the
    prompt). Runs in the caller's process."""
    L = ctypes.CDLL(REF_LIB)
    L.refh_open.restype = ctypes.c_void_p
    L.refh_open.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    h = ctypes.c_void_p(L.refh_open(path.encode(), n_prompt + nwarm + ngen + 8, threads, 1))
    if not h.value:
        raise RuntimeError("reference could not open the model")
    info = (ctypes.c_int * 8)()
    nv = L.refh_info(h, info)
    lg = np.zeros(nv, np.float32)
    lp = lg.ctypes.data_as(ctypes.c_void_p)
    prompt = np.random.default_rng(1234).integers(0, nv, n_prompt)
    tok = 0
    for i, t in enumerate(prompt):
        tok = L.refh_forward(h, int(t), i, lp)
    ids = [int(tok)]
    pos = n_prompt
    for _ in range(nwarm):
        tok = L.refh_forward(h, int(tok), pos, lp)
        ids.append(int(tok))
        pos += 1
    t0 = time.perf_counter()
    for _ in range(ngen):
        tok = L.refh_forward(h, int(tok), pos, lp)
        ids.append(int(tok))
        pos += 1
    dt = time.perf_counter() - t0
    L.refh_close(h)
    return ngen / dt, dt, ids


def _cpu_child(args):
    return cpu_decode(*args)


def cpu_decode_isolated(path, n_prompt, nwarm, ngen, threads):
    # a fresh process: the reference keeps model-format state per process
    import concurrent.futures as cf
    import multiprocessing as mp
    with cf.ProcessPoolExecutor(max_workers=1, mp_context=mp.get_context("spawn")) as ex:
        return ex.submit(_cpu_child, (path, n_prompt, nwarm, ngen, threads)).result()


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=120)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="sheep", choices=["sheep", "reference"])
    a = ap.parse_args()
    K, W = max(2, a.steps), max(3, a.warmup)

    from sheep_b200 import dist as sdist
    world, rank, local = sdist.rank_info()
    from sheep_b200 import configs
    spec = dict(configs.CONFIGS["qwen2.5-1.5b-q4"])

    if a.impl == "reference":
        # the reference's own CPU path, rank 0 only
        if rank != 0:
            return
        if not os.path.exists(REF_LIB):
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libsmlref.so was not built "
                              "(the reference tree was absent at build time)"}))
            return
        path = model_path(spec, 0, None, own_process=True)
        cores = host_cores()
        # at least 32 greedy ids (warm-up + timed) for the ids line
        wr = max(W, 32 - K)
        tps, dt, ids = cpu_decode_isolated(path, PROMPT_LEN, wr, K, cores)
        sample = f"{PROMPT_LEN}-token prompt stepped, {wr} warm-up tokens, {K} timed greedy tokens"
        print(json.dumps({
            "metric": METRIC, "value": tps, "unit": "tok/s", "n_gpus": a.gpus, "steps": K, "warmup": W,
            "ms_per_step": 1000.0 / tps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "s8xu4->s32, f32 epilogue", "data": "synthetic (seeded N(0,0.02) weights, RTN Q4)",
            "impl": "reference",
            "config": bench_config(W, K),
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": cores, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "greedy_ids_32": ids[:32],
        }))
        return

    import torch
    # NCCL's start-up banner would land on stdout beside the one JSON line
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    dist = sdist.init("nccl", timeout_s=300)
    if dist is None:
        torch.cuda.set_device(0)
    import sheep_b200
    path = model_path(spec, rank, dist)
    n_ctx = max(PROMPT_LEN + W + K + 8, PROMPT_LEN + 40)
    # N > 1: one decode stream split over the N GPUs (tensor parallelism)
    tp = (world, rank, dist) if world > 1 else None
    eng = sheep_b200.Engine(path, n_ctx=n_ctx, tp=tp)
    prompt = np.random.default_rng(1234).integers(0, eng.n_vocab, PROMPT_LEN).astype(np.int32)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        return sdist.max_over_ranks(dist, v)

    # ---- device-resident decode: K tokens after the prompt and W warm-up tokens
    ids32 = eng.generate(prompt, 32)   # the first 32 greedy ids; first replays, outside the timed region
    barrier()
    with Clocks(local) as clk:
        ids, ms = eng.generate(prompt, K + 1, timed=True, warmup=W)   # K + 1 ids = K timed replays
        barrier()
    ms = max_over_ranks(ms)
    value = K / (ms / 1000.0)
    launches = eng.launches_per_token
    bytes_rank = float(eng.bytes_per_token)

    # ---- the dominant kernel (fused gate/up GEMV, this rank's rows) alone, for the roofline
    k_ms, k_bytes = eng.time_kernel("ffn", 2 * eng.n_layer)
    barrier()

    # ---- end to end through the reference-facing API, host buffers: host ids
    # in, host logits out, host argmax (sml_gpu_step; with N GPUs its handle
    # form sb_step on every rank)
    if world == 1:
        eng.close()
        ok, why = sheep_b200.sml_gpu_open(path, n_ctx)
        if not ok:
            raise RuntimeError(why)
        # the logits as a C caller gets them: the library's host buffer, read in place
        prefill = lambda ids_, p0: sheep_b200.sml_gpu_prefill(ids_, p0)
        step = lambda t, p: sheep_b200.sml_gpu_step(t, p, copy=False)
    else:
        prefill, step = eng.prefill, eng.step
    lg = prefill(prompt, 0)
    pos = PROMPT_LEN
    for _ in range(W):
        lg = step(int(np.argmax(lg)), pos)
        pos += 1
    barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        lg = step(int(np.argmax(lg)), pos)
        pos += 1
    e2e_s = time.perf_counter() - t0
    if world == 1:
        sheep_b200.sml_gpu_close()
    else:
        eng.close()
    e2e_s = max_over_ranks(e2e_s)
    e2e = K / e2e_s
    nv = len(lg)
    bytes_all = bytes_rank
    if dist is not None:
        t = torch.tensor([bytes_rank], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        bytes_all = float(t.item())

    cpu = None
    if rank == 0 and world == 1 and os.path.exists(REF_LIB):
        cores = host_cores()
        n_cpu = 24
        tps, _, _ = cpu_decode_isolated(path, PROMPT_LEN, 2, n_cpu, cores)
        cpu = {"value": tps, "unit": "tok/s", "cores": cores, "kind": "reference",
               "sample": f"same model and prompt ({PROMPT_LEN} ids stepped), 2 warm-up then {n_cpu} timed greedy tokens"}

    extras = None
    if world > 1:
        # every rank: configuration 3 split the same way, and configuration 2's
        # MoE layer spread over the GPUs (expert parallelism, the library's NCCL
        # all-reduce between down and combine)
        peak0, _ = peaks()
        d3 = decode_cfg3(peak0, tp=(world, rank, dist), max_over_ranks=max_over_ranks)
        ep = moe_ep_microbench(peak0, dist, world, rank, max_over_ranks)
        d4 = decode_cfg4(peak0, tp=(world, rank, dist), max_over_ranks=max_over_ranks)
        if rank == 0:
            extras = {"decode_cfg3_tp": d3, "moe_cfg2_ep": ep, "decode_cfg4_tp": d4}
    if rank == 0 and world == 1:
        peak0, _ = peaks()
        from sheep_b200 import configs as cf
        extras = {"l2": "a 512 MB buffer rewritten before each timed run (decode: weights > L2)",
                  "gemv_cfg1": extra(gemv_microbench, peak0), "gemm_tc_cfg1": extra(gemm_tc_microbench, peak0),
                  "moe_cfg2": extra(moe_microbench, peak0),
                  "decode_cfg3": extra(decode_cfg3, peak0), "decode_cfg3_batch64": extra(decode_cfg3_batch, peak0),
                  "decode_cfg4": extra(decode_cfg4, peak0),
                  "decode_cfg4_batch64": extra(decode_cfg4_batch, peak0),
                  "prefill_cfg0": extra(lambda: prefill_bench(model_path(cf.CONFIGS["qwen2.5-1.5b-q4"], 0, None),
                                                              PROMPT_LEN)),
                  "prefill_cfg3": extra(lambda: prefill_bench(model_path(cf.CONFIGS["llama3-8b-q4k"], 0, None),
                                                              2048))}

    if rank == 0:
        peak, peak_kind = peaks()
        achieved = k_bytes / (k_ms / 1000.0) / 1e9
        traffic = profiled_traffic("tgemv_ffn_cfg0")
        out = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "s8xu4->s32, f32 epilogue", "data": "synthetic (seeded N(0,0.02) weights, RTN Q4)",
            "config": bench_config(W, K),
            "parallelism": ("one GPU" if world == 1 else
                            f"tp{world}: one decode stream; gate/up, down and head rows split over {world} GPUs, "
                            "attention replicated, rows exchanged over NVLink by the GEMVs"),
            "l2": "weights 0.89 GB/token > 126 MB L2: no flush",
            "roofline": {"kernel": "k_tgemv<FFN> (fused gate/up dequant-GEMV + SiLU), launched alone",
                         "bound": "hbm", "achieved": achieved, "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": achieved / peak,
                         "traffic": traffic, "algorithmic_bytes_per_launch": k_bytes,
                         "launch_us": k_ms * 1000.0},
            "token_roofline": {"bytes_per_token": float(spec_bytes(path)),
                               "achieved_gbs": float(spec_bytes(path)) / (ms / K / 1000.0) / 1e9,
                               "frac": float(spec_bytes(path)) / (ms / K / 1000.0) / 1e9 / peak,
                               "bytes_read_all_gpus": bytes_all,
                               "frac_of_n_gpus": bytes_all / (ms / K / 1000.0) / 1e9 / (peak * world)},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8 * world, "d2h_bytes_per_step": 4 * nv * world,
                    "path": "sml_gpu_step (host ids in, host logits out, host argmax)" if world == 1 else
                            "sb_step on every rank (host ids in, host logits out, host argmax)"},
            "gpu_launches": launches * K * world,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "greedy_ids_32": [int(i) for i in ids32[:32]],
            "extras": extras,
        }
        print(json.dumps(out))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def extra(fn, *args):
    """One extra measurement; a failure is reported in its place instead of
    ending the run (the headline line is printed either way)."""
    try:
        return fn(*args)
    except Exception as e:   # noqa: BLE001 -- any failure of an extra is data, not a crash
        return {"error": f"{type(e).__name__}: {e}"[:300]}


def fp16_rows(seed, n, cols):
    """fp16 N(0, 1) activations as float32 rows."""
    return np.random.default_rng(seed).standard_normal((n, cols)).astype(np.float16).astype(np.float32)


def prefill_bench(path, n_prompt, ngen=12):
    """Prompt reading: tok/s of sb_prefill over a random n_prompt-id prompt,
    stepped (prompt level 0) and in tensor-core chunks (level 2), each after one
    untimed read; and the 12 greedy ids after the prompt both ways (the
    reference server's check of a batched prompt path)."""
    import sheep_b200
    eng = sheep_b200.Engine(path, n_ctx=n_prompt + ngen + 8)
    out = {"prompt": n_prompt}
    try:
        prompt = np.random.default_rng(2048).integers(0, eng.n_vocab, n_prompt).astype(np.int32)
        ids = {}
        for level in (0, 2):
            eng.prompt_mode(level)
            eng.prefill(prompt, 0)
            t0 = time.perf_counter()
            lg = eng.prefill(prompt, 0)
            dt = time.perf_counter() - t0
            got, pos = [], n_prompt
            for _ in range(ngen):
                got.append(int(np.argmax(lg)))
                lg = eng.step(got[-1], pos)
                pos += 1
            ids[level] = got
            out[f"level{level}_tok_s"] = round(n_prompt / dt, 1)
            out[f"level{level}_ms"] = round(dt * 1000.0, 2)
        out["ids_after_prompt_equal"] = int(sum(a == b for a, b in zip(ids[0], ids[2])))
        out["ids_compared"] = ngen
    finally:
        eng.close()
    return out


def gemv_microbench(peak, reps=20):
    """Configuration 1: weight GB/s of one GEMV over B activations."""
    import sheep_b200
    from sheep_b200 import configs
    out = []
    for cfg, quant in (("gemv-4096-q4", "Q4"), ("gemv-4096-q8", "Q8")):
        ts = sheep_b200.TensorSet(model_path(configs.CONFIGS[cfg], 0, None))
        try:
            for name in ("blk.0.attn_q.weight", "blk.0.ffn_gate.weight", "blk.0.ffn_down.weight"):
                rows, cols, _ = ts.shape(name)
                nbytes = ts.nbytes(name)
                for B in (1, 4, 16):
                    ms = ts.time_gemv(name, fp16_rows(B, B, cols), reps)
                    gbs = nbytes / (ms / 1000.0) / 1e9
                    out.append({"quant": quant, "shape": f"{rows}x{cols}", "batch": B, "us": round(ms * 1000.0, 2),
                                "weight_bytes": nbytes, "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)})
        finally:
            ts.close()
    return out


def decode_cfg3(peak, ngen=64, tp=None, max_over_ranks=None):
    """Configuration 3 (Llama-3-8B shape, 6-bit group fields) at batch 1: the
    device-resident greedy loop after a 128-token prompt; with tp=(world, rank,
    dist) one stream split over the GPUs (every rank calls this)."""
    import sheep_b200
    from sheep_b200 import configs
    rank, dist = (tp[1], tp[2]) if tp else (0, None)
    path = model_path(configs.CONFIGS["llama3-8b-q4k"], rank, dist)
    eng = sheep_b200.Engine(path, n_ctx=PROMPT_LEN + 8 + ngen + 8, tp=tp)
    try:
        prompt = np.random.default_rng(1234).integers(0, eng.n_vocab, PROMPT_LEN).astype(np.int32)
        ids, ms = eng.generate(prompt, ngen + 1, timed=True, warmup=8)
        if max_over_ranks:
            ms = max_over_ranks(ms)
        tps = ngen / (ms / 1000.0)
        nb = float(eng.bytes_per_token)
        world = tp[0] if tp else 1
        if dist is not None:
            import torch
            t = torch.tensor([nb], dtype=torch.float64, device="cuda")
            dist.all_reduce(t)
            nb = float(t.item())
        gbs = nb * tps / 1e9
        return {"tok_s": round(tps, 1), "ms_per_token": round(ms / ngen, 4), "gpus": world,
                "bytes_per_token_all_gpus": int(nb), "gbs": round(gbs, 1), "frac_of_n_gpus": round(gbs / (peak * world), 4),
                "tokens": ngen, "greedy_ids_head": [int(i) for i in ids[:8]]}
    finally:
        eng.close()


def decode_cfg4(peak, prompt=1024, ngen=64, nwarm=8, tp=None, max_over_ranks=None):
    """Configuration 4 (Qwen3-235B-A22B shape, 94 MoE layers, ~136 GB of Q4)
    at batch 1: a `prompt`-id random prompt stepped, then the device-resident
    greedy loop. The file holds everything but the experts (writer mode
    direct=2); the engine draws the experts' tiles on the device
    (sb_draw_experts), so a token reads the bytes a full file would give: the
    attention projections, the router, the 8 chosen experts of every layer and
    the head. With tp=(world, rank, dist) (every rank calls this) one stream
    over the GPUs: attention replicated, each layer's experts spread over them
    (their per-choice outputs summed by NCCL), the head split by rows."""
    import sheep_b200
    from sheep_b200 import configs
    rank, dist = (tp[1], tp[2]) if tp else (0, None)
    path = model_path(configs.CONFIGS["qwen3-235b-a22b-q4"], rank, dist)
    sheep_b200.draw_experts(235)
    t0 = time.time()
    try:
        eng = sheep_b200.Engine(path, n_ctx=prompt + nwarm + ngen + 8, tp=tp)
    finally:
        sheep_b200.draw_experts(0)
    open_s = time.time() - t0
    try:
        p = np.random.default_rng(1234).integers(0, eng.n_vocab, prompt).astype(np.int32)
        ids, ms = eng.generate(p, ngen + 1, timed=True, warmup=nwarm)
        if max_over_ranks:
            ms = max_over_ranks(ms)
        tps = ngen / (ms / 1000.0)
        nb = float(eng.bytes_per_token)
        world = tp[0] if tp else 1
        if dist is not None:
            import torch
            t = torch.tensor([nb], dtype=torch.float64, device="cuda")
            dist.all_reduce(t)
            nb = float(t.item())
        gbs = nb * tps / 1e9
        return {"tok_s": round(tps, 1), "ms_per_token": round(ms / ngen, 4), "gpus": world, "prompt": prompt,
                "tokens": ngen, "bytes_per_token_all_gpus": int(nb), "gbs": round(gbs, 1),
                "frac_of_n_gpus": round(gbs / (peak * world), 4),
                "experts": "drawn on the device (direct=2 file)" + (f"; spread over {world} GPUs" if world > 1 else ""),
                "open_s": round(open_s, 1), "launches_per_token": eng.launches_per_token,
                "greedy_ids_head": [int(i) for i in ids[:8]]}
    finally:
        eng.close()


def decode_cfg3_batch(peak, n_seq=64, prompt=2048, ngen=256, nwarm=4):
    """Configuration 3 as batched serving: n_seq sequences, each a `prompt`-id
    random prompt stepped through the batched engine, then ngen greedy tokens
    per sequence decoded together (one weight read per step, every product on
    the tensor cores). Timed: the last ngen - 1 steps (CUDA events). Bytes per
    step: the weights once (the file's Q4 bytes, the metric's algorithmic
    figure, and the int8 re-quantized bytes the products actually read) plus
    every sequence's KV cache up to its position."""
    import sheep_b200
    from sheep_b200 import configs
    spec = configs.CONFIGS["llama3-8b-q4k"]
    path = model_path(spec, 0, None)
    n_ctx = prompt + nwarm + ngen
    t0 = time.time()
    b = sheep_b200.Batch(path, n_seq, n_ctx)
    t_open = time.time() - t0
    try:
        prompts = np.random.default_rng(64).integers(0, b.n_vocab, (n_seq, prompt)).astype(np.int32)
        t0 = time.time()
        ids, ms = b.generate(prompts, ngen, nwarm=nwarm, timed=True)
        t_run = time.time() - t0
        steps = ngen - 1
        tps = n_seq * steps / (ms / 1000.0)
        kv_row = spec["n_layer"] * 2 * spec["n_head_kv"] * spec["head_dim"] * 2   # bytes per position per sequence
        first = prompt + nwarm + 1                        # positions of the timed steps: first .. first + steps - 1
        kv_step = n_seq * kv_row * (first + (steps - 1) / 2.0 + 1)   # mean cached positions read per step
        alg = b.file_bytes + kv_step
        real = b.int8_bytes + kv_step
        return {"n_seq": n_seq, "prompt": prompt, "generated": ngen, "tok_s": round(tps, 1),
                "ms_per_step": round(ms / steps, 4), "bytes_per_step_alg": int(alg),
                "gbs_alg": round(alg * steps / (ms / 1000.0) / 1e9, 1),
                "frac_alg": round(alg * steps / (ms / 1000.0) / 1e9 / peak, 4),
                "bytes_per_step_read": int(real), "gbs_read": round(real * steps / (ms / 1000.0) / 1e9, 1),
                "frac_read": round(real * steps / (ms / 1000.0) / 1e9 / peak, 4),
                "splits_qkv_o_gu_down_head": b.splits, "launches_per_step": b.launches,
                "open_s": round(t_open, 1), "run_s": round(t_run, 1),
                "ids_distinct": int(len(np.unique(ids)))}
    finally:
        b.close()


def decode_cfg4_batch(peak, n_seq=64, prompt=1024, ngen=32, nwarm=2):
    """Configuration 4 as batched serving on one GPU: n_seq sequences of a
    `prompt`-id random prompt stepped through the batched engine, then ngen
    greedy tokens each decoded together: per MoE layer the router and the
    chosen experts of all n_seq rows on the tensor cores (f16, codes decoded
    in shared memory), the attention products on the int8 tensor-core path.
    Experts drawn on the device (the direct=2 file). Bytes per step: the
    attention and head weights once (as stored), every expert (at 64 rows x 8
    choices almost all of the 128 are chosen in every layer) and the KV caches
    up to each position."""
    import sheep_b200
    from sheep_b200 import configs
    spec = configs.CONFIGS["qwen3-235b-a22b-q4"]
    path = model_path(spec, 0, None)
    n_ctx = prompt + nwarm + ngen
    sheep_b200.draw_experts(235)
    t0 = time.time()
    try:
        b = sheep_b200.Batch(path, n_seq, n_ctx)
    finally:
        sheep_b200.draw_experts(0)
    t_open = time.time() - t0
    try:
        prompts = np.random.default_rng(65).integers(0, b.n_vocab, (n_seq, prompt)).astype(np.int32)
        t0 = time.time()
        ids, ms = b.generate(prompts, ngen, nwarm=nwarm, timed=True)
        t_run = time.time() - t0
        steps = ngen - 1
        tps = n_seq * steps / (ms / 1000.0)
        kv_row = spec["n_layer"] * 2 * spec["n_head_kv"] * spec["head_dim"] * 2
        first = prompt + nwarm + 1
        kv_step = n_seq * kv_row * (first + (steps - 1) / 2.0 + 1)
        alg = b.file_bytes + b.expert_bytes + kv_step
        return {"n_seq": n_seq, "prompt": prompt, "generated": ngen, "tok_s": round(tps, 1),
                "ms_per_step": round(ms / steps, 3), "bytes_per_step_alg": int(alg),
                "gbs_alg": round(alg * steps / (ms / 1000.0) / 1e9, 1),
                "frac_alg": round(alg * steps / (ms / 1000.0) / 1e9 / peak, 4),
                "experts": "drawn on the device (direct=2 file); expert products on the tensor cores",
                "launches_per_step": b.launches, "open_s": round(t_open, 1), "run_s": round(t_run, 1)}
    finally:
        b.close()


def gemm_tc_microbench(peak, reps=20):
    """Configuration 1's matrices at 16/64/256 rows of x on the tensor cores
    (the batched path's int8 arithmetic): TOPS of the int8 products and GB/s
    of the re-quantized int8 weights read."""
    import sheep_b200
    from sheep_b200 import configs
    out = []
    for cfg, quant in (("gemv-4096-q4", "Q4"), ("gemv-4096-q8", "Q8")):
        ts = sheep_b200.TensorSet(model_path(configs.CONFIGS[cfg], 0, None))
        try:
            for name in ("blk.0.attn_q.weight", "blk.0.ffn_gate.weight", "blk.0.ffn_down.weight"):
                rows, cols, _ = ts.shape(name)
                for B in (16, 64, 256):
                    ms = ts.time_gemm_tc(name, fp16_rows(B, B, cols), reps)
                    w8 = rows * ((cols // 32 + 7) // 8) * 256
                    out.append({"quant": quant, "shape": f"{rows}x{cols}", "batch": B, "us": round(ms * 1000.0, 2),
                                "int8_tops": round(2.0 * rows * cols * B / (ms / 1000.0) / 1e12, 1),
                                "int8_weight_gbs": round(w8 / (ms / 1000.0) / 1e9, 1)})
        finally:
            ts.close()
    return out


def moe_ep_microbench(peak, dist, world, rank, max_over_ranks, reps=20):
    """Configuration 2's MoE layer over `world` GPUs (expert parallelism): every
    rank holds 128/world experts. Two exchanges: "all-reduce" (every rank
    passes all T tokens, the per-choice outputs summed over the GPUs) and
    "all-to-all" (each rank passes T/world tokens of its own, rows sent to the
    GPUs holding their experts and back). Timed per rank by CUDA events with L2
    flushed, the max over ranks reported. Bytes: the chosen experts summed over
    the ranks (each rank reads only those it holds) plus every rank's router."""
    import sheep_b200
    from sheep_b200 import configs
    from sheep_b200 import dist as sdist
    nid = sdist.share_nccl_id(dist)
    m = sheep_b200.MoeLayer(model_path(configs.CONFIGS["qwen3-30b-a3b-moe-layer"], 0, None), max_tokens=256,
                            ep=(world, rank, nid))
    out = []
    try:
        import torch
        for mode in ("all-reduce", "all-to-all"):
            m.exchange(mode)
            for T in (1, 16, 64, 256):
                if mode == "all-to-all" and T < world:
                    continue
                # all-to-all: this rank's share of the T tokens (rows of the same seeded set)
                x = fp16_rows(100 + T, T, m.n_embd)
                if mode == "all-to-all":
                    x = x[T * rank // world:T * (rank + 1) // world]
                ms, na = m.time(x, reps)
                ms = max_over_ranks(ms)
                t = torch.tensor([float(na)], dtype=torch.float64, device="cuda")
                if dist is not None:
                    dist.all_reduce(t)
                na_all = int(t.item())
                nbytes = na_all * m.expert_bytes + world * m.router_bytes
                gbs = nbytes / (ms / 1000.0) / 1e9
                out.append({"exchange": mode, "tokens": T, "gpus": world, "us": round(ms * 1000.0, 2),
                            "tok_s": round(T / (ms / 1000.0), 1), "experts_read": na_all, "bytes": nbytes,
                            "gbs": round(gbs, 1), "frac_of_n_gpus": round(gbs / (peak * world), 4)})
    finally:
        m.close()
    return out


def moe_microbench(peak, reps=20):
    """Configuration 2: the MoE layer at T tokens a step."""
    import sheep_b200
    from sheep_b200 import configs
    m = sheep_b200.MoeLayer(model_path(configs.CONFIGS["qwen3-30b-a3b-moe-layer"], 0, None), max_tokens=256)
    out = []
    try:
        for T in (1, 16, 64, 256):
            # 16+ rows: both paths (the default picks the tensor cores from 8
            # chosen rows per expert on average: here 128 rows)
            for tc in ((True, False) if T >= 16 else (False,)):
                m.tensor_cores(tc)
                ms, na = m.time(fp16_rows(100 + T, T, m.n_embd), reps)
                nbytes = na * m.expert_bytes + m.router_bytes
                gbs = nbytes / (ms / 1000.0) / 1e9
                out.append({"tokens": T, "path": "tensor cores (f16)" if tc else "integer (dp4a)",
                            "us": round(ms * 1000.0, 2), "tok_s": round(T / (ms / 1000.0), 1),
                            "experts_read": na, "bytes": nbytes, "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)})
            m.tensor_cores("auto")
    finally:
        m.close()
    return out


def spec_bytes(path):
    """Weight bytes one token reads: every quantized record's codes and fields
    (the tied embedding counted once, as the head)."""
    import struct
    tot = 0
    with open(path, "rb") as f:
        head = f.read(4096)
        n, toff = struct.unpack_from("<QQ", head, 68)
        f.seek(toff)
        raw = f.read(n * 248)
    for i in range(n):
        v = struct.unpack_from("<64s4I2Q2Q2Q2Q2Q2Q4Q4Q2I", raw, i * 248)
        kind = v[1]
        if kind != 1:
            continue
        sd_n, sq_n, md_n, mq_n = v[8], v[10], v[14], v[16]
        codes = sum(v[21:25])
        tot += sd_n + sq_n + md_n + mq_n + codes
    return tot


if __name__ == "__main__":
    main()
