"""Write the golden vectors in tests/golden/ from the reference's own CPU code.

Run in a container that has the reference tree (oracle/_ref/libsmlref.so built
by oracle/Makefile from its unchanged sources):

    python tests/golden/make_golden.py

For every flat width Q2..Q8 with 8-bit and 6-bit group fields, a one-layer
synthetic model (its spec and the file's sha256 recorded, so the writer is
pinned too) and, computed by the reference (sml_quantize_act, the per-width
matvec dispatch of sml-run.c, the sml_dequant_row_* functions):
  - the int8 activation of sml-check's deterministic input, gathered;
  - y = W x for two tensors;
  - three dequantized embedding rows.
For a two-layer model: 8 greedy ids after an 8-token prompt and their logits
(sml_forward, the prompt stepped a token at a time). The same for a two-layer
mixture-of-experts model (16 experts, 4 per token, renormalized softmax), and
sml_moe_route's choices and weights on seeded logits with planted ties, for
moe_flags 1 and 0. sml_quantize_act_sb's per-256 activation (the batched
path's) on seeded vectors with a zero superblock, exact .5 ties, saturation
and a partial last superblock.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

WIDTHS = [(nb, six) for six in (0, 1) for nb in (2, 3, 4, 5, 6, 7, 8)]
PROMPT = [3, 1, 4, 1, 5, 9, 2, 6]


def width_spec(nb, six):
    import sheep_b200
    return sheep_b200.spec_for("tiny-q4", n_layer=1, nbits=nb, emb_nbits=nb, scale6=six, minneg=six,
                               seed=500 + 10 * nb + six, tied=0)


def decode_spec():
    import sheep_b200
    return sheep_b200.spec_for("tiny-q4", seed=77)


def moe_spec():
    import sheep_b200
    return sheep_b200.spec_for("tiny-q4", seed=91, n_expert=16, n_expert_used=4, moe_flags=1, expert_ff=384)


def route_logits():
    rng = np.random.default_rng(2024)
    lg = rng.standard_normal((24, 128)).astype(np.float32)
    for t in range(0, 24, 3):                    # ties: the lower index wins
        lg[t, rng.integers(0, 128, 6)] = lg[t].max()
    lg[1, :] = 0.5                               # every expert tied
    return lg


def act_sb_inputs():
    rng = np.random.default_rng(77)
    xs = []
    for n in (256, 1024, 1408, 4096):      # 1408: a partial (4-group) last superblock
        x = rng.standard_normal(n).astype(np.float32)
        xs.append(x)
    x = np.zeros(1408, np.float32)
    x[256:512] = np.float32(0.5) * np.arange(256, dtype=np.float32) - 64.0   # .5 ties at amax 63.5 -> 127/63.5 = 2
    x[512:768] = 127.0
    x[513] = -1e6                                                             # one huge value: everything else rounds to 0
    x[1280:] = rng.standard_normal(128).astype(np.float32) * 1e-30            # tiny, still nonzero
    xs.append(x)
    return xs


def check_input(n):
    """sml/sml-check.c:194: x[i] = sin(0.001 i) * (1 + 0.5 (i % 7))."""
    i = np.arange(n, dtype=np.float32)
    return (np.sin(np.float32(0.001) * i) * (np.float32(1.0) + np.float32(0.5) * (i % 7).astype(np.float32))).astype(np.float32)


TENSORS = ("blk.0.ffn_down.weight", "output.weight")


def main():
    from tests import helpers
    assert helpers.have_ref(), "needs oracle/_ref/libsmlref.so (build it with `make -C oracle ref`)"
    index = {}
    for nb, six in WIDTHS:
        spec = width_spec(nb, six)
        path = helpers.model_path(spec)
        recs = helpers.read_records(path)
        out = {}
        for t in TENSORS:
            rows, cols = recs[t]["rows"], recs[t]["cols"]
            x = check_input(cols)
            y, q, s, sums = helpers.ref("matvec", path, name=t, x=x, rows=rows)
            key = t.replace(".", "_")
            out[key + "_y"] = y
            out[key + "_q"] = q
            out[key + "_s"] = s
            out[key + "_sums"] = sums
        r = recs["token_embd.weight"]
        rows = [0, 5, r["rows"] - 1]
        out["embd_rows"] = np.array(rows, np.int32)
        out["embd_deq"] = helpers.ref("dequant", path, name="token_embd.weight", rows=rows, cols=r["cols"])
        name = f"width_q{nb}_f{8 if not six else 6}.npz"
        np.savez_compressed(os.path.join(HERE, name), **out)
        index[name] = {"spec": spec, "sha256": helpers.file_sha(path)}
    spec = decode_spec()
    path = helpers.model_path(spec)
    ids, lg = helpers.ref("decode", path, prompt=PROMPT, ngen=8, n_ctx=64)
    np.savez_compressed(os.path.join(HERE, "decode_tiny.npz"), ids=ids, logits=lg, prompt=np.array(PROMPT, np.int32))
    index["decode_tiny.npz"] = {"spec": spec, "sha256": helpers.file_sha(path)}
    spec = moe_spec()
    path = helpers.model_path(spec)
    ids, lg = helpers.ref("decode", path, prompt=PROMPT, ngen=8, n_ctx=64)
    np.savez_compressed(os.path.join(HERE, "decode_moe_tiny.npz"), ids=ids, logits=lg,
                        prompt=np.array(PROMPT, np.int32))
    index["decode_moe_tiny.npz"] = {"spec": spec, "sha256": helpers.file_sha(path)}
    lgs = route_logits()
    out = {"logits": lgs}
    for flags in (1, 0):
        sel = np.zeros((len(lgs), 8), np.int32)
        w = np.zeros((len(lgs), 8), np.float32)
        for t in range(len(lgs)):
            sel[t], w[t] = helpers.ref("route", lg=lgs[t], k=8, flags=flags)
        out[f"sel_f{flags}"] = sel
        out[f"w_f{flags}"] = w
    np.savez_compressed(os.path.join(HERE, "route.npz"), **out)
    out = {}
    for i, x in enumerate(act_sb_inputs()):
        q, s, sums = helpers.ref("quant_sb", x=x)
        out[f"x{i}"], out[f"q{i}"], out[f"s{i}"], out[f"sums{i}"] = x, q, s, sums
    np.savez_compressed(os.path.join(HERE, "act_sb.npz"), **out)
    index["act_sb.npz"] = {"inputs": len(act_sb_inputs())}
    index["route.npz"] = {"k": 8, "n_expert": 128}
    with open(os.path.join(HERE, "index.json"), "w") as f:
        json.dump(index, f, indent=1, sort_keys=True)
    print("wrote", len(index), "fixtures")


if __name__ == "__main__":
    main()
