"""llmq_run, the reference CLI's `llama` subcommand (main.c:624-702) on the
GPU path: the same stdin/stdout protocol and the same ids as the reference's
loop (token-by-token decode, sample_token with temperature 0.8, top-k 40,
top-p 0.95, one stream seeded 1234 for the whole run), which the test replays
with the oracle's decode and sampler."""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, ROOT
from helpers import fp, orc_sample

CLI = os.path.join(ROOT, "llm-project_b200", "bin", "llmq_run")
MODEL = os.path.join(GOLDEN, "mini.llmq")


def reference_protocol(orc, lines, n_new):
    """main.c:650-671 over the oracle: returns the stdout lines."""
    import llmq
    m = llmq.QLlamaModel()
    assert orc.orc_model_load(MODEL.encode(), C.byref(m)) == 0
    state = 0x4D2  # rng_create(1234)
    out = []
    row = np.zeros(m.vocab, np.float32)
    for line in lines:
        if line.startswith("\ufeff"):
            line = line[1:]
        seq = []
        for t in line.split():  # main.c:562-572: out-of-range ids are skipped, at most max_seq kept
            if len(seq) == m.max_seq:
                break
            if 0 <= int(t) < m.vocab:
                seq.append(int(t))
        if not seq:
            continue
        kv = orc.orc_kv_create(C.byref(m))
        for t in seq:
            orc.orc_decode_step(C.byref(m), C.byref(kv), t, fp(row))
        n = len(seq)
        for _ in range(n_new):
            if n >= m.max_seq:
                break
            nxt, state = orc_sample(orc, row, 0.8, 40, 0.95, state)
            seq.append(nxt)
            n += 1
            out.append(f"t {nxt}")
            orc.orc_decode_step(C.byref(m), C.byref(kv), nxt, fp(row))
        out.append("gen: " + " ".join(str(i) for i in seq))
        orc.orc_kv_free(C.byref(kv))
    orc.orc_model_free(C.byref(m))
    return out


def test_cli_built():
    assert os.access(CLI, os.X_OK), "build with make -C llm-project_b200/csrc"


def test_cli_usage_and_bad_checkpoint(tmp_path):
    r = subprocess.run([CLI], capture_output=True, text=True)
    assert r.returncode == 2 and "usage" in r.stderr
    r = subprocess.run([CLI, "llama"], capture_output=True, text=True)
    assert r.returncode == 2
    bad = tmp_path / "f32.bin"
    bad.write_bytes(b"LLMA" + b"\0" * 60)
    r = subprocess.run([CLI, "llama", str(bad)], capture_output=True, text=True, input="1 2\n")
    assert r.returncode == 1 and "LLMA (f32)" in r.stderr


@pytest.mark.gpu
def test_cli_matches_reference_loop(orc):
    rng = np.random.default_rng(17)
    long_prompt = " ".join(str(i) for i in rng.integers(0, 512, 300))
    lines = ["3 141 59 26 5", "\ufeff7 600 8 9", "", "   ", long_prompt, "42"]
    n_new = 24
    want = reference_protocol(orc, lines, n_new)
    stdin = "".join(l + "\n" for l in lines)
    r = subprocess.run([CLI, "llama", MODEL, str(n_new)], input=stdin, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.splitlines() == want
    assert "skip out-of-range id 600 (vocab 512)" in r.stderr
    assert "loaded LLMQ (int8, in-memory): vocab 512" in r.stderr
