"""The reference's own server (sml/sml-server.c, unchanged) linked against
libsheep_b200.so in place of the reference's GPU library (oracle/Makefile,
_ref/sml-server): the real caller of the drop-in boundary.

On the GPU the server opens the model with sml_gpu_open, runs its prompt-path
probe (sml/sml-server.c:1625-1680: 12 greedy ids after a prompt read stepped,
then through sml_gpu_prefill at levels 2 and 1, keeping the first level whose
ids agree), then serves OpenAI chat requests through fwd_prefill / fwd_step
(:217-259): sml_gpu_prefill at absolute positions after the cached prefix the
slot already holds, sml_gpu_step per generated token. The tests check the
replies against this repository's engine making the same calls.

The synthetic models get a small vocabulary (tests/helpers.with_vocab): the
letters a-z are its byte tokens, every other id reads "[id]", so a reply's text
gives back its ids exactly.
"""
import json
import os
import socket
import subprocess
import time
import urllib.request

import numpy as np
import pytest

import sheep_b200
from tests import helpers

SERVER = os.path.join(helpers.ORACLE_DIR, "_ref", "sml-server")

needs_server = pytest.mark.skipif(not os.path.exists(SERVER),
                                  reason="oracle/_ref/sml-server was not built (needs the reference tree)")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class Server:
    """sml-server on a model, one device, a free loopback port."""

    def __init__(self, path, device, n_ctx=256):
        self.port = _free_port()
        self.log = open(path + f".{device}.log", "w")
        env = dict(os.environ)
        env["SML_PROMPT_RECHECK"] = "1"   # probe the prompt path on this box, never from a stale record
        self.p = subprocess.Popen([SERVER, path, "--device", device, "--port", str(self.port), "--ctx", str(n_ctx),
                                   "--threads", "4", "--orchestrator", "off"],
                                  stdout=self.log, stderr=subprocess.STDOUT, env=env)
        t0 = time.time()
        while True:
            if self.p.poll() is not None:
                raise RuntimeError(f"sml-server exited with {self.p.returncode}: {open(self.log.name).read()[-2000:]}")
            try:
                if self.get("/health")["status"] == "ok":
                    break
            except OSError:
                pass
            if time.time() - t0 > 120:
                raise RuntimeError("sml-server did not start listening")
            time.sleep(0.2)

    def get(self, route):
        with urllib.request.urlopen(f"http://127.0.0.1:{self.port}{route}", timeout=60) as r:
            return json.loads(r.read())

    def chat(self, prompt, max_tokens):
        """A raw prompt (taken as is), greedy, no response cache: (ids, reply)."""
        body = json.dumps({"prompt": prompt, "max_tokens": max_tokens, "temperature": 0, "cache": False}).encode()
        req = urllib.request.Request(f"http://127.0.0.1:{self.port}/v1/chat/completions", data=body,
                                     headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=120) as r:
            rep = json.loads(r.read())
        return helpers.vocab_ids(rep["choices"][0]["message"]["content"]), rep

    def close(self):
        if self.p.poll() is None:
            self.p.terminate()
            try:
                self.p.wait(timeout=30)
            except subprocess.TimeoutExpired:
                self.p.kill()
                self.p.wait()
        self.log.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def _ids(text):
    return [helpers.VOCAB_LETTERS.index(c) for c in text]


@needs_server
def test_server_serves_on_the_cpu():
    """The server reads the synthetic vocabulary and answers a request (its
    own CPU engine): one prompt id per letter, max_tokens ids back."""
    path = helpers.with_vocab(helpers.model_path(sheep_b200.spec_for("tiny-q4")))
    with Server(path, "cpu") as srv:
        ids, rep = srv.chat("thequickbrownfox", 8)
        st = srv.get("/stats")
    assert rep["usage"]["prompt_tokens"] == len("thequickbrownfox")
    assert rep["usage"]["completion_tokens"] == len(ids) == 8
    assert st["device"] == "cpu" and st["template"] == "plain"


def _engine_replay(path, level, turns):
    """The server's calls for each (prompt ids, reused, n) turn on a fresh
    engine: sml_gpu_prefill of the ids past the reused prefix at their
    absolute positions, then n greedy steps (first index of the largest
    logit, as sml_sample_greedy)."""
    eng = sheep_b200.Engine(path, n_ctx=256)
    out = []
    try:
        eng.prompt_mode(level)
        for ids, reused, n in turns:
            lg = eng.prefill(np.array(ids[reused:], np.int32), reused)
            pos, got = len(ids), []
            for _ in range(n):
                got.append(int(np.argmax(lg)))
                lg = eng.step(got[-1], pos)
                pos += 1
            out.append(got)
    finally:
        eng.close()
    return out


@needs_server
@pytest.mark.gpu
@pytest.mark.parametrize("spec", [
    dict(name="tiny-q4"),
    dict(name="tiny-q4", n_layer=4, qkv_bias=1, seed=21),
])
def test_server_on_the_gpu_matches_the_engine(spec):
    """sml-server serving on the GPU through this library: the probe picks a
    prompt level, two turns of one conversation (the second continues the
    first, so the server reuses the cached prefix and reads only the new ids
    at their absolute positions), and every generated id equals this
    repository's engine making the same calls."""
    s = dict(spec)
    path = helpers.with_vocab(helpers.model_path(sheep_b200.spec_for(s.pop("name"), **s)))
    p1, p2_more = "thequickbrownfoxjumpsoverthelazydog", "andrunsaway"
    with Server(path, "gpu") as srv:
        st = srv.get("/stats")
        ids1, rep1 = srv.chat(p1, 12)
        ids2, rep2 = srv.chat(p1 + p2_more, 12)
    with open(path + ".prompt") as f:
        level = int(f.read().split()[-1])
    assert st["device"] == "gpu" and st["gpu_layers"] == st["gpu_of"] > 0, st
    assert rep1["sml"]["reused"] == 0
    reused = rep2["sml"]["reused"]
    assert reused >= len(p1), rep2["sml"]   # at least the first prompt is the slot's prefix
    assert len(ids1) == rep1["usage"]["completion_tokens"] > 0
    assert len(ids2) == rep2["usage"]["completion_tokens"] > 0
    want1, want2 = _engine_replay(path, level, [(_ids(p1), 0, len(ids1)),
                                                (_ids(p1 + p2_more), reused, len(ids2))])
    print(f"prompt level {level}; turn 1 {ids1}; turn 2 (reused {reused}) {ids2}")
    assert ids1 == want1
    assert ids2 == want2
