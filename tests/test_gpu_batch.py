"""Batched serving on the GPU (sb_batch_*, the reference's sml_forward_multi)
against the CPU restatement of the same arithmetic (so_batch mode 1: every
product on the batched path's int8 arithmetic, attention/norms/RoPE per
sequence), and against the decode arithmetic (mode 0) for the spread the
batched arithmetic itself costs (the reference's `sml-batched --check` figures:
max|dlogit|/max|logit| and greedy agreement, sml/sml-batched.c:95-137)."""
import numpy as np
import pytest

import sheep_b200
from tests import helpers

pytestmark = pytest.mark.gpu


def _model(**over):
    spec = sheep_b200.spec_for("tiny-q4", **over)
    return helpers.model_path(spec)


# ---------------------------------------------------------------- split-K products

@pytest.mark.parametrize("split", [2, 3, 4])
def test_gemm_tc_split_matches_restatement(split):
    """Superblock slices summed in slice order equal the restatement bit for bit."""
    path = _model(n_embd=1024, n_ff=2816, n_head=8, n_head_kv=2, head_dim=128, n_layer=1, seed=41)
    ts = sheep_b200.TensorSet(path)
    orc = helpers.Oracle(path)
    rng = np.random.default_rng(split)
    try:
        for name in ("blk.0.ffn_down.weight", "blk.0.attn_q.weight", "output.weight"):
            rows, cols, _ = ts.shape(name)
            nsb = (cols // 32 + 7) // 8
            per = -(-nsb // split)
            if -(-nsb // per) != split:
                continue
            for T in (16, 40, 64):
                X = rng.standard_normal((T, cols)).astype(np.float16).astype(np.float32)
                Y = ts.gemm_tc(name, X, split=split)
                Yo = orc.gemm_sb_split(name, X, rows, split)
                assert np.array_equal(Y.view(np.uint32), Yo.view(np.uint32)), (name, T, split)
    finally:
        ts.close()
        orc.close()


def test_gemm_tc_split_rejects_empty_slices():
    path = _model(n_embd=512, n_layer=1, seed=42)
    ts = sheep_b200.TensorSet(path)
    try:
        rows, cols, _ = ts.shape("blk.0.attn_q.weight")   # 2 superblocks
        X = np.ones((16, cols), np.float32)
        with pytest.raises(RuntimeError):
            ts.gemm_tc("blk.0.attn_q.weight", X, split=3)
    finally:
        ts.close()


# ---------------------------------------------------------------- the batched step

def _drive(path, n_seq, steps, np_, starts, n_ctx=64, seed=0, kv_check=0):
    """Step the GPU batch and both CPU restatements with the same tokens: prompt
    ids while a slot's position is inside its prompt, then the GPU's greedy
    choice. Returns per step (active mask, gpu logits, batched-arith logits,
    decode-arith logits). kv_check (the KV row width): every layer-0 cache row
    written is compared bit for bit with the restatement's."""
    rng = np.random.default_rng(seed)
    b = sheep_b200.Batch(path, n_seq, n_ctx)
    orc = helpers.Oracle(path, n_ctx)
    ob1 = helpers.OracleBatch(orc, n_seq, 1, b.splits)
    ob0 = helpers.OracleBatch(orc, n_seq, 0)
    prompts = rng.integers(0, b.n_vocab, (n_seq, np_)).astype(np.int32)
    last = np.zeros(n_seq, np.int32)
    out = []
    try:
        for t in range(steps):
            pos = np.array([t - s for s in starts], np.int32)
            pos[pos < 0] = -1
            tok = np.where(pos < 0, 0, np.where(pos < np_, prompts[np.arange(n_seq), np.clip(pos, 0, np_ - 1)], last))
            tok = tok.astype(np.int32)
            lg = b.forward_multi(tok, pos)
            l1 = ob1.step(tok, pos)
            l0 = ob0.step(tok, pos)
            act = pos >= 0
            if kv_check:
                for s in np.nonzero(act)[0]:
                    kg, vg = b.kv(0, s, pos[s], kv_check)
                    ko, vo = ob1.kv(0, s, pos[s], kv_check)
                    assert np.array_equal(kg, ko) and np.array_equal(vg, vo), (t, s)
            last = np.where(act, lg.argmax(1), last).astype(np.int32)
            out.append((act, lg, l1, l0))
    finally:
        ob1.close()
        ob0.close()
        orc.close()
        b.close()
    return out


def _spread(out):
    r1, agree1, rms0, ratio0, agree0 = [], 0, 0.0, 0.0, 0
    for act, lg, l1, l0 in out:
        for s in np.nonzero(act)[0]:
            r1.append(helpers.rel_rms(l1[s], lg[s]))
            rms0 = max(rms0, helpers.rel_rms(l0[s], lg[s]))
            ratio0 = max(ratio0, float(np.abs(l0[s] - lg[s]).max() / (np.abs(l0[s]).max() + 1e-9)))
            agree1 += int(l1[s].argmax() == lg[s].argmax())
            agree0 += int(l0[s].argmax() == lg[s].argmax())
    r1 = np.array(r1)
    return r1, agree1, rms0, ratio0, agree0, len(r1)


BATCH_MODELS = [
    # (spec overrides, slots)
    (dict(seed=51), 20),                                                          # hd 64, GQA 2, q/k/v bias
    (dict(n_embd=512, n_head=8, n_head_kv=2, head_dim=128, n_ff=1408, seed=52), 17),   # hd 128, GQA 4
    (dict(n_embd=768, n_head=12, n_head_kv=2, head_dim=64, n_ff=1536, tied=1, qk_norm=1, seed=53), 33),
    (dict(nbits=6, emb_nbits=6, scale6=1, minneg=1, seed=54), 16),               # v9 6-bit fields
    (dict(nbits=6, emb_nbits=6, seed=54), 16),                                   # 6-bit codes, 8-bit fields
]


@pytest.mark.parametrize("over,n_seq", BATCH_MODELS)
def test_batch_matches_restatement(over, n_seq):
    """Every active slot, step by step over ragged positions and idle slots
    (prompt ids, then greedy), against the CPU restatement of the batched
    arithmetic:
      - layer 0's cached keys and values bit-equal (embedding, norm, int8
        products, bias, RoPE and fp16 rounding all the same arithmetic);
      - logits: 80 % of slot-steps within 1e-5 rel-RMS, all within 3e-2,
        greedy ids equal on 97 %. Attention sums its floats in another order
        (a few ulps apart); when that flips one int8 code of the next product's
        input, the slot's later steps move to the quantization's own noise,
        ~1e-2. Reproduced on the CPU: the restatement with +-2 to 8 ulps of
        noise on its attention outputs moves 11-30 of 280 slot-steps, by up to
        1.3e-2 -- the spread seen here;
    and against the decode arithmetic within the batched arithmetic's own
    spread (int8 weights at 1/127 of a superblock's range, activations per 256)."""
    path = _model(**over)
    spec = sheep_b200.spec_for("tiny-q4", **over)
    starts = [s % 5 for s in range(n_seq)]
    out = _drive(path, n_seq, steps=14, np_=5, starts=starts, seed=n_seq,
                 kv_check=spec["n_head_kv"] * spec["head_dim"])
    r1, agree1, rms0, ratio0, agree0, n = _spread(out)
    print(f"slots {n_seq}: vs batched arithmetic rel-RMS median {np.median(r1):.1e} p80 {np.quantile(r1, 0.8):.1e} "
          f"max {r1.max():.2e} moved {(r1 > 1e-5).sum()}/{n} agree {agree1}/{n}; vs decode arithmetic rel-RMS "
          f"{rms0:.2e} max|d|/max {ratio0:.2e} agree {agree0}/{n}")
    assert np.quantile(r1, 0.8) <= 1e-5, np.quantile(r1, 0.8)
    assert r1.max() <= 3e-2, r1.max()
    assert agree1 >= int(0.97 * n), (agree1, n)
    assert rms0 <= 6e-2, rms0
    assert agree0 >= int(0.8 * n), (agree0, n)


@pytest.mark.skipif(not helpers.have_ref(), reason="reference CPU build (oracle/_ref) not present")
def test_batch_against_reference_forward_multi():
    """The GPU batch against the reference's own multi-conversation step
    (sml_forward_multi, oracle/_ref): eight conversations, ragged starts and
    idle slots, teacher-forced ids. Against both of its arithmetics -- the
    default for more than two conversations (per-256 activations on the 4-bit
    codes, sml/sml-run.c:2579-2597) and SML_MULTI=exact (the decode kernels) --
    every slot-step within the batched arithmetic's spread and greedy ids
    mostly equal (the reference's sml-batched --check measures the same two
    quantities, sml/sml-batched.c:95-137)."""
    path = _model(seed=61)
    ns, nsteps, starts = 8, 10, [0, 1, 2, 3, 0, 5, 1, 2]
    toks = np.random.default_rng(12).integers(0, 1024, (nsteps, ns)).astype(np.int32)
    steps = [(toks[t].tolist(), [t - s if t >= s else -1 for s in starts]) for t in range(nsteps)]
    ref_sb = helpers.ref("multi", path, ns=ns, n_vocab=1024, steps=steps, n_ctx=32)
    ref_ex = helpers.ref("multi", path, ns=ns, n_vocab=1024, steps=steps, n_ctx=32, env={"SML_MULTI": "exact"})
    with sheep_b200.Batch(path, ns, 32) as b:
        got = [b.forward_multi(np.array(tok, np.int32), np.array(pos, np.int32)) for tok, pos in steps]
    for name, ref in (("per-256", ref_sb), ("exact", ref_ex)):
        rms, agree, n = [], 0, 0
        for t, (tok, pos) in enumerate(steps):
            for s in range(ns):
                if pos[s] >= 0:
                    rms.append(helpers.rel_rms(ref[t][s], got[t][s]))
                    agree += int(np.argmax(ref[t][s]) == np.argmax(got[t][s]))
                    n += 1
        print(f"vs reference {name}: rel-RMS median {np.median(rms):.2e} max {max(rms):.2e} greedy {agree}/{n}")
        assert max(rms) <= 6e-2, (name, max(rms))
        assert agree >= int(0.8 * n), (name, agree, n)


@pytest.mark.skipif(not helpers.have_ref(), reason="reference CPU build (oracle/_ref) not present")
def test_batch_moe_against_reference_forward_multi():
    """Mixture-of-experts layers on the batched path (two layers of 16
    experts, top-4, Q/K norm): every row through the router and its chosen
    experts (the decode arithmetic per row), the attention side on the tensor
    cores. Against the reference's own sml_forward_multi in both arithmetics
    (its batched step runs moe_ffn_batch, sml/sml-run.c:3182): eight
    conversations, ragged starts and idle slots, every slot-step within the
    batched arithmetic's spread and greedy ids mostly equal; two GPU runs
    bit-identical."""
    spec = sheep_b200.spec_for("tiny-q4", n_expert=16, n_expert_used=4, moe_flags=1, expert_ff=384, qk_norm=1,
                               seed=93)
    path = helpers.model_path(spec)
    ns, nsteps, starts = 8, 10, [0, 1, 2, 3, 0, 5, 1, 2]
    toks = np.random.default_rng(14).integers(0, 1024, (nsteps, ns)).astype(np.int32)
    steps = [(toks[t].tolist(), [t - s if t >= s else -1 for s in starts]) for t in range(nsteps)]
    ref_sb = helpers.ref("multi", path, ns=ns, n_vocab=1024, steps=steps, n_ctx=32)
    ref_ex = helpers.ref("multi", path, ns=ns, n_vocab=1024, steps=steps, n_ctx=32, env={"SML_MULTI": "exact"})
    runs = []
    for _ in range(2):
        with sheep_b200.Batch(path, ns, 32) as b:
            assert b.expert_bytes > 0
            runs.append([b.forward_multi(np.array(tok, np.int32), np.array(pos, np.int32)) for tok, pos in steps])
    got = runs[0]
    for t in range(nsteps):
        for s in range(ns):
            if steps[t][1][s] >= 0:
                assert np.array_equal(got[t][s].view(np.uint32), runs[1][t][s].view(np.uint32)), (t, s)
    # the reference's own spread between its two arithmetics on these steps:
    # the GPU may differ from either by about as much (its products mix them:
    # per-256 attention products, per-32 expert products)
    spread = max(helpers.rel_rms(ref_ex[t][s], ref_sb[t][s])
                 for t, (tok, pos) in enumerate(steps) for s in range(ns) if pos[s] >= 0)
    bound = max(6e-2, 1.5 * spread)
    print(f"reference per-256 vs exact: max rel-RMS {spread:.2e}; bound {bound:.2e}")
    for name, ref in (("per-256", ref_sb), ("exact", ref_ex)):
        rms, agree, n = [], 0, 0
        for t, (tok, pos) in enumerate(steps):
            for s in range(ns):
                if pos[s] >= 0:
                    rms.append(helpers.rel_rms(ref[t][s], got[t][s]))
                    agree += int(np.argmax(ref[t][s]) == np.argmax(got[t][s]))
                    n += 1
        print(f"MoE vs reference {name}: rel-RMS median {np.median(rms):.2e} max {max(rms):.2e} greedy {agree}/{n}")
        assert max(rms) <= bound, (name, max(rms), bound)
        assert agree >= int(0.8 * n), (name, agree, n)


def test_batch_deterministic():
    """Two runs of the same steps give the same logits bit for bit (split sums
    and chunk combines in a fixed order, never in arrival order)."""
    path = _model(n_embd=512, n_head=8, n_head_kv=2, head_dim=128, n_ff=1408, seed=59)
    rng = np.random.default_rng(9)
    toks = rng.integers(0, 1024, (40, 24)).astype(np.int32)
    runs = []
    for _ in range(2):
        with sheep_b200.Batch(path, 24, 160) as b:
            for t in range(40):
                lg = b.forward_multi(toks[t], np.full(24, t * 4, np.int32))   # two chunks of 128 by the end
            runs.append(lg)
    assert np.array_equal(runs[0].view(np.uint32), runs[1].view(np.uint32))


def test_batch_long_context_chunks():
    """Positions across three 128-position chunks (partials combined by the
    last CTA of each sequence and KV head): the same bar against the
    restatement. Positions jump; both sides read never-written cache rows as
    zeros, so the histories stay identical."""
    path = _model(n_embd=512, n_head=8, n_head_kv=2, head_dim=128, n_ff=1408, seed=60)
    n_seq = 16
    sched = [0, 1, 2, 3, 126, 127, 128, 129, 254, 255, 256, 257, 300, 301]
    rng = np.random.default_rng(10)
    toks = rng.integers(0, 1024, (len(sched), n_seq)).astype(np.int32)
    b = sheep_b200.Batch(path, n_seq, 320)
    orc = helpers.Oracle(path, 320)
    ob1 = helpers.OracleBatch(orc, n_seq, 1, b.splits)
    r1 = []
    try:
        for t, p in enumerate(sched):
            pos = np.full(n_seq, p, np.int32)
            pos[::3] = -1 if t % 2 else p   # some slots idle on odd steps
            lg = b.forward_multi(toks[t], pos)
            l1 = ob1.step(toks[t], pos)
            r1 += [helpers.rel_rms(l1[s], lg[s]) for s in range(n_seq) if pos[s] >= 0]
    finally:
        ob1.close()
        orc.close()
        b.close()
    r1 = np.array(r1)
    print(f"long context: rel-RMS median {np.median(r1):.1e} p95 {np.quantile(r1, 0.95):.1e} max {r1.max():.2e}")
    # the batched attention sums in another order than the reference's (whose
    # order the restatement keeps): over 300-position rows more slot-steps see
    # a last-bit difference flip an int8 code; the majority stay at the
    # restatement's last bits and none leaves the quantization's noise
    assert np.median(r1) <= 1e-5
    assert r1.max() <= 3e-2


def test_batch_slots_independent():
    """A slot's logits do not depend on what the other slots hold (each token's
    products, quantization and attention are its own): bit-equal across batches
    that differ elsewhere, and with the other slots idle."""
    path = _model(seed=55)
    rng = np.random.default_rng(5)
    n_seq = 24
    prompt = rng.integers(0, 1024, 6).astype(np.int32)
    results = []
    for variant in range(3):
        b = sheep_b200.Batch(path, n_seq, 32)
        try:
            others = rng.integers(0, 1024, (n_seq, 6)).astype(np.int32)
            for t in range(6):
                tok = others[:, t].copy()
                tok[7] = prompt[t]
                pos = np.full(n_seq, t, np.int32) if variant < 2 else np.full(n_seq, -1, np.int32)
                pos[7] = t
                lg = b.forward_multi(tok, pos)
            results.append(lg[7].copy())
        finally:
            b.close()
    assert np.array_equal(results[0].view(np.uint32), results[1].view(np.uint32))
    assert np.array_equal(results[0].view(np.uint32), results[2].view(np.uint32))


def test_batch_generate_equals_stepping():
    """Device-side greedy generation (graph replays, ids fed back on the GPU)
    gives the ids of stepping forward_multi with the host taking the argmax."""
    path = _model(seed=56)
    rng = np.random.default_rng(6)
    n_seq, np_, ngen = 18, 5, 9
    prompts = rng.integers(0, 1024, (n_seq, np_)).astype(np.int32)
    with sheep_b200.Batch(path, n_seq, 32) as b:
        ids = b.generate(prompts, ngen, nwarm=2)
    with sheep_b200.Batch(path, n_seq, 32) as b:
        for i in range(np_):
            lg = b.forward_multi(prompts[:, i], np.full(n_seq, i, np.int32))
        ref = []
        for g in range(ngen + 2):
            tok = lg.argmax(1).astype(np.int32)
            ref.append(tok)
            if g + 1 < ngen + 2:
                lg = b.forward_multi(tok, np.full(n_seq, np_ + g, np.int32))
    assert np.array_equal(ids, np.stack(ref, 1))


def test_batch_bad_args():
    path = _model(seed=57)
    with sheep_b200.Batch(path, 16, 32) as b:
        with pytest.raises(RuntimeError):
            b.forward_multi(np.zeros(16, np.int32), np.full(16, 32, np.int32))     # position == n_ctx
        with pytest.raises(RuntimeError):
            b.forward_multi(np.full(16, 5000, np.int32), np.zeros(16, np.int32))   # id >= n_vocab
        lg = b.forward_multi(np.zeros(16, np.int32), np.zeros(16, np.int32))       # still usable
        assert np.isfinite(lg).all()
        with pytest.raises(RuntimeError):
            b.generate(np.zeros((16, 30), np.int32), 4)                            # past n_ctx
    moe = helpers.model_path(sheep_b200.spec_for("tiny-q4", n_expert=8, n_expert_used=2, expert_ff=256,
                                                 moe_flags=2, seed=58))
    with pytest.raises(RuntimeError, match="routing"):
        sheep_b200.Batch(moe, 16, 32)                                          # sigmoid routing: refused by name
