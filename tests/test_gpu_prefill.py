"""Prompt reading on the tensor cores (sb_prefill at prompt level 2, the
reference's gpu_prefill with its tensor-core product): all but the last prompt
token in chunks of up to 64 through the batched arithmetic, the last stepped.

The bar is the reference server's own check of a batched prompt path
(sml/sml-server.c:1625-1680, prompt_path_sound :1050-1063): 12 greedy ids
after the prompt, read in batches, must equal those after the prompt stepped a
token at a time, or at least agree on the first 4 and not be stuck repeating
one word. Level 0 must equal stepping bit for bit."""
import numpy as np
import pytest

import sheep_b200
from tests import helpers

pytestmark = pytest.mark.gpu


def _sound(want, got):
    if list(want) == list(got):
        return True
    if list(want[:4]) != list(got[:4]):
        return False
    vals, counts = np.unique(got, return_counts=True)
    return counts.max() <= 4 and len(vals) >= 5


def _after_prompt(eng, prompt, level, ngen=12):
    eng.prompt_mode(level)
    lg = eng.prefill(prompt, 0)
    first = lg.copy()
    ids = []
    pos = len(prompt)
    for _ in range(ngen):
        t = int(np.argmax(lg))
        ids.append(t)
        lg = eng.step(t, pos)
        pos += 1
    return np.array(ids), first


MODELS = [
    ("tiny-q4", {}),
    ("small-q4-tied", {}),
    ("qwen2.5-1.5b-q4", dict(n_layer=2, n_vocab=32768, tied=0, seed=22)),   # configuration 0's widths
]


@pytest.mark.parametrize("cfg,over", MODELS)
def test_prefill_tensor_cores_reads_what_stepping_reads(cfg, over):
    spec = sheep_b200.spec_for(cfg, **over)
    path = helpers.model_path(spec)
    rng = np.random.default_rng(70)
    prompt = rng.integers(0, spec["n_vocab"], 70).astype(np.int32)   # chunks of 64 and 5, then the last
    eng = sheep_b200.Engine(path, n_ctx=128)
    try:
        want, lg0 = _after_prompt(eng, prompt, 0)
        got, lg2 = _after_prompt(eng, prompt, 2)
        # level 0 is stepping itself
        again, lg0b = _after_prompt(eng, prompt, 0)
    finally:
        eng.close()
    assert np.array_equal(lg0.view(np.uint32), lg0b.view(np.uint32)) and np.array_equal(want, again)
    print(f"{cfg}: stepped {want.tolist()} batched {got.tolist()} rel-RMS {helpers.rel_rms(lg0, lg2):.2e}")
    assert helpers.rel_rms(lg0, lg2) <= 6e-2
    assert _sound(want, got), (want, got)


def test_prefill_level0_equals_stepping_bit_for_bit():
    path = helpers.model_path(sheep_b200.spec_for("small-q4-tied"))
    prompt = np.random.default_rng(71).integers(0, 4096, 20).astype(np.int32)
    eng = sheep_b200.Engine(path, n_ctx=64)
    try:
        eng.prompt_mode(0)
        lp = eng.prefill(prompt, 0)
        ls = None
        for i, t in enumerate(prompt):
            ls = eng.step(int(t), i)
    finally:
        eng.close()
    assert np.array_equal(lp.view(np.uint32), ls.view(np.uint32))


def test_prefill_continues_a_cached_prefix():
    """Absolute positions continue the cache (sml/sml-gpu.h:14): a prompt read
    as a prefix then a suffix at pos0 gives what one read of the whole gives."""
    path = helpers.model_path(sheep_b200.spec_for("tiny-q4"))
    prompt = np.random.default_rng(72).integers(0, 1024, 90).astype(np.int32)
    eng = sheep_b200.Engine(path, n_ctx=128)
    try:
        eng.prompt_mode(2)
        whole = eng.prefill(prompt, 0)
        eng.prefill(prompt[:50], 0)
        parts = eng.prefill(prompt[50:], 50)
    finally:
        eng.close()
    # the prefix's last token is stepped in the two-part read but read in a chunk
    # in the whole one: the same up to the batched arithmetic's noise
    assert helpers.rel_rms(whole, parts) <= 6e-2
    assert int(np.argmax(whole)) == int(np.argmax(parts)) or helpers.agree_with_ties(whole, parts)[0]


@pytest.mark.parametrize("cfg,over", [("tiny-q4", {}), ("small-q4-tied", dict(qk_norm=1))])
def test_prefill_cache_rows_equal_batched_restatement(cfg, over):
    """The chunk path is the batched arithmetic exactly: the cache rows it
    writes equal the CPU restatement's (so_batch mode 1: the same int8 products
    with the same superblock slices, the same per-256 activations, the
    reference-order attention) bit for bit -- every layer of a prompt read in
    two chunks, and layer 0 of a continuation at pos0."""
    spec = sheep_b200.spec_for(cfg, **over)
    path = helpers.model_path(spec)
    prompt = np.random.default_rng(73).integers(0, spec["n_vocab"], 75).astype(np.int32)
    eng = sheep_b200.Engine(path, n_ctx=96)
    try:
        eng.prompt_mode(2)
        splits = eng.prompt_splits()
        eng.prefill(prompt[:67], 0)      # rows 0..65 in chunks of 64 and 2, 66 stepped
        eng.prefill(prompt[67:], 67)     # rows 67..73 in one chunk, 74 stepped
        kvd = spec["n_head_kv"] * spec["head_dim"]
        got = {(l, p): eng.kv_rows(l, p) for l in range(spec["n_layer"]) for p in range(75)}
    finally:
        eng.close()
    orc = helpers.Oracle(path, 96)
    ob = helpers.OracleBatch(orc, 1, 1, splits)
    try:
        for p, t in enumerate(prompt):
            ob.step(np.array([t], np.int32), np.array([p], np.int32))
        # rows 66 and 74 the decode arithmetic wrote (the restatement writes them
        # in the batched one); a later row of layer >= 1 attends to row 66 of
        # the layer below, so past it only layer 0 (the token's own row) compares
        for l in range(spec["n_layer"]):
            for p in range(75):
                if p in (66, 74) or (l > 0 and p > 66):
                    continue
                k, v = ob.kv(l, 0, p, kvd)
                assert np.array_equal(got[(l, p)][0], k) and np.array_equal(got[(l, p)][1], v), (l, p)
    finally:
        ob.close()
        orc.close()
