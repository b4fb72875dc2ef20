"""Continuous batching over the paged KV cache (sb_batch_open_paged,
sb_forward_seqs): sequences take pages of 64 positions from a shared pool as
they grow, join and leave the step between any two steps, run in whatever
slot is free, and give their pages back when freed.

The bar: a sequence's logits at every step, and its cached rows, equal bit for
bit those of the same sequence decoded alone in a fixed slot of the slot-form
engine (sb_forward_multi with the same number of slots), whatever its slot,
its pages or the other sequences of the step -- each slot's products,
quantization and attention are its own (the reference's sml_forward_multi
gives each conversation its own context, sml/sml-run.c:2559-2604).
"""
import numpy as np
import pytest

import sheep_b200
from tests import helpers

pytestmark = pytest.mark.gpu

MODELS = [
    dict(seed=61),                                                                # hd 64 (tensor-core attention)
    dict(n_embd=512, n_head=8, n_head_kv=2, head_dim=128, n_ff=1408, seed=62),    # hd 128, GQA 4
    dict(n_embd=512, n_head=4, n_head_kv=2, head_dim=256, n_ff=1024, seed=63),    # hd 256 (CUDA-core attention)
]


def _model(**over):
    return helpers.model_path(sheep_b200.spec_for("tiny-q4", **over))


def _alone(path, n_slots, n_ctx, prompt, ngen, kv_at, kvd):
    """One sequence in slot 0 of the slot-form engine, the other slots idle:
    the logits of every step, its greedy ids, and its cached rows at kv_at."""
    out, ids = [], []
    with sheep_b200.Batch(path, n_slots, n_ctx) as b:
        tok = int(prompt[0])
        for pos in range(len(prompt) + ngen):
            t = np.zeros(n_slots, np.int32)
            p = np.full(n_slots, -1, np.int32)
            t[0], p[0] = tok, pos
            lg = b.forward_multi(t, p)[0]
            out.append(lg)
            if pos + 1 < len(prompt):
                tok = int(prompt[pos + 1])
            else:
                tok = int(np.argmax(lg))
                ids.append(tok)
        kv = {q: b.kv(0, 0, q, kvd) for q in kv_at}
    return out, ids, kv


@pytest.mark.parametrize("over", MODELS)
def test_paged_continuous_batching_equals_alone(over):
    """Six sequences through four slots and a pool too small to hold them all:
    admitted as pages allow, rotated across the slots every step, freed when
    done (their pages reused by later ones). Every step's logits, the greedy
    ids and the cached rows (at page edges too) equal each sequence decoded
    alone, bit for bit."""
    path = _model(**over)
    spec = sheep_b200.spec_for("tiny-q4", **over)
    kvd = spec["n_head_kv"] * spec["head_dim"]
    n_slots, n_ctx, n_pages, ngen = 4, 192, 7, 8
    rng = np.random.default_rng(7)
    lens = [70, 130, 40, 100, 64, 90]
    prompts = [rng.integers(0, 1024, n).astype(np.int32) for n in lens]
    need = [(n + ngen + 63) // 64 for n in lens]
    assert sum(need) > n_pages
    # cached rows at page edges and the last position (those the sequence reached)
    ref = [_alone(path, n_slots, n_ctx, p, ngen, sorted({q for q in (0, 63, 64, len(p) + ngen - 1)
                                                         if q < len(p) + ngen}), kvd) for p in prompts]

    got = [[] for _ in lens]
    gids = [[] for _ in lens]
    with sheep_b200.PagedBatch(path, n_slots, n_ctx, n_pages) as pb:
        assert pb.pages() == (n_pages, n_pages, 0)
        waiting, active, reserved, step = list(range(len(lens))), [], 0, 0
        seq_of, pos_of, tok_of = {}, {}, {}
        kv_seen = {}
        while waiting or active:
            # admit in order while slots and the pages a sequence will reach allow
            while waiting and len(active) < n_slots and reserved + need[waiting[0]] <= n_pages:
                i = waiting.pop(0)
                seq_of[i], pos_of[i], tok_of[i] = pb.new_seq(), 0, int(prompts[i][0])
                reserved += need[i]
                active.append(i)
            order = active[step % len(active):] + active[:step % len(active)]   # a new slot every step
            lg = pb.forward([seq_of[i] for i in order], [tok_of[i] for i in order], [pos_of[i] for i in order])
            for s, i in enumerate(order):
                got[i].append(lg[s])
                pos = pos_of[i]
                if pos + 1 < lens[i]:
                    tok_of[i] = int(prompts[i][pos + 1])
                else:
                    tok_of[i] = int(np.argmax(lg[s]))
                    gids[i].append(tok_of[i])
                pos_of[i] = pos + 1
                if pos_of[i] == lens[i] + ngen:
                    kv_seen[i] = {q: pb.kv(0, seq_of[i], q, kvd) for q in ref[i][2]}
                    pb.free_seq(seq_of[i])
                    active.remove(i)
                    reserved -= need[i]
            step += 1
        assert pb.pages() == (n_pages, n_pages, 0)
    for i in range(len(lens)):
        want, wids, wkv = ref[i]
        assert len(got[i]) == len(want)
        for t, (a, b) in enumerate(zip(got[i], want)):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (i, t)
        assert gids[i] == wids
        for q, (k, v) in wkv.items():
            assert np.array_equal(kv_seen[i][q][0], k) and np.array_equal(kv_seen[i][q][1], v), (i, q)


def test_paged_truncate_continues_like_fresh():
    """A sequence cut back to 50 positions (its second page returned) and fed
    new ids from there equals a fresh sequence fed the same 50 ids and the new
    ones (the server's prefix reuse)."""
    path = _model(seed=64)
    rng = np.random.default_rng(8)
    a_ids = rng.integers(0, 1024, 100).astype(np.int32)
    more = rng.integers(0, 1024, 30).astype(np.int32)
    with sheep_b200.PagedBatch(path, 2, 128, 6) as pb:
        a = pb.new_seq()
        for pos, t in enumerate(a_ids):
            pb.forward([a], [t], [pos])
        assert pb.pages()[1] == 4
        pb.truncate(a, 50)
        assert pb.pages()[1] == 5
        out_a = [pb.forward([a], [t], [50 + j])[0] for j, t in enumerate(more)]
        c = pb.new_seq()
        seq = np.concatenate([a_ids[:50], more])
        out_c = [pb.forward([c], [t], [pos])[0] for pos, t in enumerate(seq)][50:]
    for x, y in zip(out_a, out_c):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32))


def test_paged_pool_exhausted_changes_nothing():
    """A step whose sequences need more pages than are free fails and leaves
    every table as it was; freeing a sequence makes room."""
    path = _model(seed=65)
    with sheep_b200.PagedBatch(path, 2, 128, 2) as pb:
        a, b = pb.new_seq(), pb.new_seq()
        pb.forward([a], [1], [0])
        pb.forward([a], [2], [64])
        assert pb.pages() == (2, 0, 2)
        with pytest.raises(RuntimeError, match="pages"):
            pb.forward([a, b], [3, 4], [65, 0])
        assert pb.pages() == (2, 0, 2)
        pb.free_seq(a)
        assert pb.pages() == (2, 2, 1)
        pb.forward([b], [4], [0])
        assert pb.pages() == (2, 1, 1)


def test_paged_refusals():
    path = _model(seed=66)
    with sheep_b200.PagedBatch(path, 2, 128, 4) as pb:
        a = pb.new_seq()
        with pytest.raises(RuntimeError, match="two slots"):
            pb.forward([a, a], [1, 2], [0, 0])
        with pytest.raises(RuntimeError, match="not live"):
            pb.forward([a + 1], [1], [0])
        with pytest.raises(RuntimeError, match="out of range"):
            pb.forward([a], [1], [128])
        with pytest.raises(RuntimeError, match="bad arguments"):
            pb.forward([a, a, a], [1, 1, 1], [0, 1, 2])     # more sequences than slots
        pb.free_seq(a)
        with pytest.raises(RuntimeError, match="not live"):
            pb.forward([a], [1], [0])
        # the slot-form calls refuse a paged handle
        t = np.zeros(2, np.int32)
        assert not sheep_b200.lib().sb_forward_multi(pb.h, helpers._p(t), helpers._p(t))
