"""Sampler parity (sampler.c:8-115): the oracle restatement against the
reference build on the CPU, then the GPU sampler (standalone sample_token /
sample_argmax, and fused into the decode graph) against both.  The bar is the
same token id and the same xorshift64 state after every draw."""
from __future__ import annotations

import ctypes as C
import math

import numpy as np
import pytest

import llmq
from helpers import (SAMPLER_SETTINGS, TINY, fp, orc_sample, ref_sample, sampler_k, sampler_rows, synth)

DRAWS = 4
SEEDS = [1234, 0, 0xFFFFFFFFFFFFFFFF]


def start_state(lib_or_ref, seed: int) -> int:
    return lib_or_ref.rng_create(seed).state


# ---------------------------------------------------------------- CPU only
def test_rng_stream_matches_reference(lib, ref):
    """rng_create / rng_uniform (host code in libllmq_cuda.so) give the
    reference's stream value for value (sampler.c:26-44)."""
    for seed in SEEDS + [1, 42]:
        a, b = lib.rng_create(seed), ref.rng_create(seed)
        assert a.state == b.state
        for _ in range(2000):
            ua, ub = lib.rng_uniform(C.byref(a)), ref.rng_uniform(C.byref(b))
            assert np.float32(ua).view(np.uint32) == np.float32(ub).view(np.uint32)
            assert a.state == b.state


def test_oracle_sampler_matches_reference(orc, ref):
    """The oracle's sampler against the reference's, every row x setting,
    several chained draws: same id and same stream state."""
    rows = sampler_rows()
    for name, row in rows.items():
        for (T, k, p) in SAMPLER_SETTINGS:
            so = sr = start_state(ref, SEEDS[0])
            for d in range(DRAWS if row.size < 100000 else 2):
                to, so = orc_sample(orc, row, T, k, p, so)
                tr, sr = ref_sample(ref, row, T, k, p, sr)
                assert (to, so) == (tr, sr), (name, T, k, p, d)


def test_windowed_chain_sum_matches_sequential_loop(tmp_path):
    """The GPU sampler's windowed evaluation of the softmax denominator
    (llmq_sample.cuh), restated on the CPU in tests/sampler_chain_check.c,
    equals the sequential float loop bit for bit on random rows of eight
    kinds (ties, subnormals, dyadic values, wide ranges)."""
    import os
    import subprocess
    src = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sampler_chain_check.c")
    exe = str(tmp_path / "chain_check")
    subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-o", exe, src, "-lm"], check=True)
    r = subprocess.run([exe, "600", "20000000"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr


def test_reference_sort_is_stable_on_ties(ref):
    """The premise of the tie rule: with all logits equal, the reference's
    top-k keeps the k lowest indices and top-p the lowest-index prefix
    (glibc's qsort is a stable merge sort)."""
    row = np.zeros(5000, np.float32)
    st = start_state(ref, 7)
    seen_k, seen_p = [], []
    for _ in range(400):
        t, st = ref_sample(ref, row, 0.8, 40, 1.0, st)
        seen_k.append(t)
        t, st = ref_sample(ref, row, 0.8, 0, 0.5, st)
        seen_p.append(t)
    assert max(seen_k) < 40 and max(seen_p) < 2500


# --------------------------------------------------------------------- GPU
def gpu_sample(lib, row, T, k, p, state):
    t = llmq.host_tensor(row.reshape(1, -1))
    r = llmq.Rng(state)
    tok = lib.sample_token(C.byref(t), 0, T, k, p, C.byref(r))
    return tok, r.state


@pytest.mark.gpu
def test_device_sample_token_matches_reference(lib, ref):
    rows = sampler_rows()
    checked = refused = 0
    for name, row in rows.items():
        for (T, k, p) in SAMPLER_SETTINGS:
            greedy = T <= 0.0
            supported = greedy or sampler_k(row.size, k) <= 1024
            for seed in SEEDS[:2]:
                sg = sr = start_state(ref, seed)
                for d in range(DRAWS):
                    if not supported:
                        tg, sg2 = gpu_sample(lib, row, T, k, p, sg)
                        assert tg == -1 and sg2 == sg and lib.q_llama_last_error() == llmq.LLMQ_ERR_ARG
                        lib.q_llama_clear_error()
                        refused += 1
                        break
                    tg, sg = gpu_sample(lib, row, T, k, p, sg)
                    tr, sr = ref_sample(ref, row, T, k, p, sr)
                    assert (tg, sg) == (tr, sr), (name, T, k, p, seed, d)
                    checked += 1
    assert checked > 300 and refused > 0


@pytest.mark.gpu
def test_device_sample_argmax_matches_reference(lib, ref):
    rows = sampler_rows()
    for name, row in rows.items():
        t = llmq.host_tensor(row.reshape(1, -1))
        assert lib.sample_argmax(C.byref(t), 0) == ref.sample_argmax(C.byref(t), 0), name
    # a later row of a 2-D tensor
    m = np.random.default_rng(3).normal(0, 1, (3, 999)).astype(np.float32)
    t = llmq.host_tensor(m)
    for r in range(3):
        assert lib.sample_argmax(C.byref(t), r) == int(np.argmax(m[r]))
        st1, st2 = llmq.Rng(99), llmq.Rng(99)
        assert lib.sample_token(C.byref(t), r, 0.7, 40, 0.9, C.byref(st1)) == \
            ref.sample_token(C.byref(t), r, 0.7, 40, 0.9, C.byref(st2))
        assert st1.state == st2.state


def orc_sampled_run(orc, ref, m, token, n, T, k, p, seed):
    """The reference CLI loop (main.c:663-668) on the oracle: decode, sample
    with the reference sampler, feed the sample back."""
    kv = orc.orc_kv_create(C.byref(m))
    row = np.zeros(m.vocab, np.float32)
    st = start_state(ref, seed)
    ids, logits = [], []
    tok = token
    for _ in range(n):
        orc.orc_decode_step(C.byref(m), C.byref(kv), tok, fp(row))
        tok, st = ref_sample(ref, row, T, k, p, st)
        ids.append(tok)
        logits.append(row.copy())
    orc.orc_kv_free(C.byref(kv))
    return ids, st, np.stack(logits)


@pytest.mark.gpu
@pytest.mark.parametrize("T,k,p", [(0.8, 40, 0.95), (1.3, 1024, 0.9), (0.0, 40, 0.95)])
def test_decode_step_sample_matches_reference_loop(lib, orc, ref, T, k, p):
    m = synth(lib, TINY, seed=1234, with_bias=True)
    n = 24
    ids_o, st_o, logits_o = orc_sampled_run(orc, ref, m, 11, n, T, k, p, 1234)
    kv = lib.q_llama_kv_create(C.byref(m))
    r = lib.rng_create(1234)
    row = np.zeros((1, m.vocab), np.float32)
    t = llmq.host_tensor(row)
    tok, ids = 11, []
    for i in range(n):
        tok = lib.q_llama_decode_step_sample(C.byref(m), C.byref(kv), tok, T, k, p, C.byref(r), C.byref(t))
        llmq.check(lib)
        assert np.array_equal(row[0].view(np.uint32), logits_o[i].view(np.uint32)), i
        ids.append(tok)
    assert ids == ids_o and r.state == st_o and kv.len == n
    lib.llama_kv_free(C.byref(kv))
    lib.q_llama_model_free(C.byref(m))


@pytest.mark.gpu
def test_generate_sample_matches_reference_loop(lib, orc, ref):
    m = synth(lib, TINY, seed=99)
    n, T, k, p = 48, 0.8, 40, 0.95
    ids_o, st_o, _ = orc_sampled_run(orc, ref, m, 3, n, T, k, p, 1234)
    kv = lib.q_llama_kv_create(C.byref(m))
    r = lib.rng_create(1234)
    out = (C.c_int * n)()
    assert lib.q_llama_generate_sample(C.byref(m), C.byref(kv), 3, n, T, k, p, C.byref(r), out) == 0
    assert list(out) == ids_o and r.state == st_o and kv.len == n
    # and in two halves: the stream carries over between calls
    kv2 = lib.q_llama_kv_create(C.byref(m))
    r2 = lib.rng_create(1234)
    a, b = (C.c_int * 20)(), (C.c_int * (n - 20))()
    assert lib.q_llama_generate_sample(C.byref(m), C.byref(kv2), 3, 20, T, k, p, C.byref(r2), a) == 0
    assert lib.q_llama_generate_sample(C.byref(m), C.byref(kv2), a[19], n - 20, T, k, p, C.byref(r2), b) == 0
    assert list(a) + list(b) == ids_o and r2.state == st_o
    # unsupported top-k: an error, nothing advanced
    r3 = lib.rng_create(5)
    s3 = r3.state
    assert lib.q_llama_generate_sample(C.byref(m), C.byref(kv2), 3, 4, 1.0, 0, 0.9, C.byref(r3), out) != 0
    assert r3.state == s3 and kv2.len == n
    lib.q_llama_clear_error()
    lib.llama_kv_free(C.byref(kv))
    lib.llama_kv_free(C.byref(kv2))
    lib.q_llama_model_free(C.byref(m))


@pytest.mark.gpu
def test_sampled_decode_8b_vocab(lib, orc, ref):
    """The 8B vocabulary (128256 logits, 32 ring chunks of the sequential sum)
    through the fused graph."""
    cfg = dict(vocab=128256, d_model=512, n_layers=2, n_heads=8, n_kv=2, head_dim=64, d_ff=1536,
               max_seq=64, rope_base=500000.0, eps=1e-5)
    m = synth(lib, cfg, seed=4321, stddev=0.5)
    n, T, k, p = 12, 0.8, 40, 0.95
    ids_o, st_o, _ = orc_sampled_run(orc, ref, m, 128000, n, T, k, p, 1234)
    kv = lib.q_llama_kv_create(C.byref(m))
    r = lib.rng_create(1234)
    out = (C.c_int * n)()
    assert lib.q_llama_generate_sample(C.byref(m), C.byref(kv), 128000, n, T, k, p, C.byref(r), out) == 0
    assert list(out) == ids_o and r.state == st_o
    lib.llama_kv_free(C.byref(kv))
    lib.q_llama_model_free(C.byref(m))
