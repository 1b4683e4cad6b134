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


def reference_protocol(orc, lines, n_new, f32_model=None):
    """main.c:650-671 (or, for an fp32 model, main.c:685-697) over the
    oracle: returns the stdout lines."""
    import llmq
    if f32_model is None:
        m = llmq.QLlamaModel()
        assert orc.orc_model_load(MODEL.encode(), C.byref(m)) == 0
        kv_create, step = orc.orc_kv_create, orc.orc_decode_step
    else:
        m = f32_model
        kv_create, step = orc.orc_f32_kv_create, orc.orc_f32_decode_step
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
        kv = kv_create(C.byref(m))
        for t in seq:
            step(C.byref(m), C.byref(kv), t, fp(row))
        n = len(seq)
        for _ in range(n_new):
            if n >= m.max_seq:
                break
            nxt, state = orc_sample(orc, row, 0.8, 40, 0.95, state)
            seq.append(nxt)
            n += 1
            out.append(f"t {nxt}")
            step(C.byref(m), C.byref(kv), nxt, fp(row))
        out.append("gen: " + " ".join(str(i) for i in seq))
        orc.orc_kv_free(C.byref(kv))
    if f32_model is None:
        orc.orc_model_free(C.byref(m))
    return out


def test_cli_built():
    assert os.access(CLI, os.X_OK), "build with make -C llm-project_b200/csrc"


def test_cli_usage_and_bad_checkpoint(tmp_path):
    r = subprocess.run([CLI], capture_output=True, text=True)
    assert r.returncode == 2 and "usage" in r.stderr
    r = subprocess.run([CLI, "llama"], capture_output=True, text=True)
    assert r.returncode == 2
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"XXXX" + b"\0" * 60)
    r = subprocess.run([CLI, "llama", str(bad)], capture_output=True, text=True, input="1 2\n")
    assert r.returncode == 1 and "not an LLMA/LLMQ checkpoint" in r.stderr
    trunc = tmp_path / "trunc.bin"
    trunc.write_bytes(b"LLMA" + b"\0" * 60)
    r = subprocess.run([CLI, "llama", str(trunc)], capture_output=True, text=True, input="1 2\n")
    assert r.returncode == 1


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


@pytest.mark.gpu
def test_cli_llma_checkpoint_matches_reference_loop(orc, ref, tmp_path):
    """An LLMA (f32) checkpoint, written by the reference's llama_model_save,
    through the fp32 GPU path."""
    import llmq
    ref.llama_model_save.restype = C.c_int
    ref.llama_model_save.argtypes = [C.c_char_p, C.POINTER(llmq.LlamaModel)]
    m = ref.llama_model_create(512, 64, 2, 4, 2, 16, 160, 48, 10000.0, 1e-5)
    ref.llama_model_randomize(C.byref(m))
    path = tmp_path / "model_f32.bin"
    assert ref.llama_model_save(str(path).encode(), C.byref(m)) == 0
    lines = ["3 141 59 26 5", "42 7", "1 2 3 4 5 6 7 8 9 10 11 12 13 14 15 16 17 18 19 20 21 22 23 24 25 26 27 28 29 30"]
    want = reference_protocol(orc, lines, 16, f32_model=m)
    r = subprocess.run([CLI, "llama", str(path), "16"], input="".join(l + "\n" for l in lines),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.splitlines() == want
    assert "loaded LLMA (f32): vocab 512" in r.stderr
    ref.llama_model_free(C.byref(m))
