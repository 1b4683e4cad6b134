"""GPU parity of the multi-row passes (batched decode and prefill) against the
oracle restatement: every row must equal the single-sequence decode step of
the reference (llama.c:528-600) bit for bit, with the products on the tcgen05
tensor-core GEMM."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import llmq
from helpers import TINY, bits_equal, gpu_decode, orc_decode, synth

pytestmark = pytest.mark.gpu

SMALL = dict(vocab=512, d_model=64, n_layers=2, n_heads=4, n_kv=2, head_dim=16, d_ff=160, max_seq=1100,
             rope_base=10000.0, eps=1e-5)


def batch_step(lib, m, kvs, tokens):
    B = len(kvs)
    out = np.full((B, m.vocab), np.nan, np.float32)
    t = llmq.host_tensor(out)
    lib.q_llama_decode_batch(C.byref(m), llmq.kv_pointers(kvs), llmq.int_array(tokens), B, C.byref(t))
    llmq.check(lib)
    return out


def new_kv(lib, m):
    kv = lib.q_llama_kv_create(C.byref(m))
    llmq.check(lib)
    return kv


def free_all(lib, m, kvs):
    for kv in kvs:
        lib.llama_kv_free(C.byref(kv))
    lib.q_llama_model_free(C.byref(m))


@pytest.mark.parametrize("cfg,with_bias", [(TINY, True), (SMALL, False)])
def test_decode_batch_matches_oracle(lib, orc, cfg, with_bias):
    """Sequences at different positions (one empty), 4 batched steps."""
    m = synth(lib, cfg, seed=99, with_bias=with_bias)
    rng = np.random.default_rng(7)
    lens = [0, 3, 11, 1, 6]
    steps = 4
    seqs = [rng.integers(0, cfg["vocab"], n + steps).tolist() for n in lens]
    kvs = [new_kv(lib, m) for _ in lens]
    for kv, s, n in zip(kvs, seqs, lens):
        if n:
            gpu_decode(lib, m, s[:n], kv=kv)
    got = np.stack([batch_step(lib, m, kvs, [s[n + i] for s, n in zip(seqs, lens)]) for i in range(steps)], axis=1)
    assert [kv.len for kv in kvs] == [n + steps for n in lens]
    for b, (s, n) in enumerate(zip(seqs, lens)):
        want, _ = orc_decode(orc, m, s)
        assert bits_equal(got[b], want[n:]), f"sequence {b}"
    free_all(lib, m, kvs)


def test_decode_batch_argmax_two_row_blocks(lib):
    """130 sequences (two 128-row tensor-core blocks): ids and logits equal the
    single-sequence GPU path, which the other tests pin to the oracle."""
    m = synth(lib, SMALL, seed=5)
    rng = np.random.default_rng(11)
    B = 130
    firsts = rng.integers(0, SMALL["vocab"], B)
    kvs = [new_kv(lib, m) for _ in range(B)]
    for kv, t in zip(kvs, firsts[:, None].tolist()):
        gpu_decode(lib, m, t, kv=kv)
    toks = rng.integers(0, SMALL["vocab"], B)
    ids = (C.c_int * B)()
    rc = lib.q_llama_decode_batch_argmax(C.byref(m), llmq.kv_pointers(kvs), llmq.int_array(toks), B, ids)
    assert rc == 0, lib.q_llama_last_error_message()
    want_ids = []
    for b in range(B):
        lg, _ = gpu_decode(lib, m, [int(firsts[b]), int(toks[b])])
        want_ids.append(int(np.argmax(lg[1])))
    assert list(ids) == want_ids
    assert all(kv.len == 2 for kv in kvs)
    free_all(lib, m, kvs)


@pytest.mark.parametrize("cfg,n,with_bias", [(TINY, 37, True), (SMALL, 1030, False), (SMALL, 1, False)])
def test_prefill_matches_oracle(lib, orc, cfg, n, with_bias):
    """Prefill of n ids (1030: two passes) gives the logits of the n-th step and
    the same cache: the following single steps match the oracle too."""
    m = synth(lib, cfg, seed=21, with_bias=with_bias)
    rng = np.random.default_rng(n)
    ids = rng.integers(0, cfg["vocab"], n + 3).tolist()
    want, _ = orc_decode(orc, m, ids)
    kv = new_kv(lib, m)
    row = np.full((1, m.vocab), np.nan, np.float32)
    t = llmq.host_tensor(row)
    nxt = lib.q_llama_prefill_argmax(C.byref(m), C.byref(kv), llmq.int_array(ids[:n]), n, C.byref(t))
    llmq.check(lib)
    assert kv.len == n
    assert bits_equal(row[0], want[n - 1])
    assert nxt == int(np.argmax(want[n - 1]))
    after, _ = gpu_decode(lib, m, ids[n:], kv=kv)
    assert bits_equal(after, want[n:])
    free_all(lib, m, [kv])


def test_prefill_continues_a_cache(lib, orc):
    """A prefill that starts at position 5 of a cache filled by single steps."""
    m = synth(lib, TINY, seed=4)
    ids = np.random.default_rng(3).integers(0, TINY["vocab"], 30).tolist()
    want, _ = orc_decode(orc, m, ids)
    kv = new_kv(lib, m)
    gpu_decode(lib, m, ids[:5], kv=kv)
    row = np.zeros((1, m.vocab), np.float32)
    lib.q_llama_prefill(C.byref(m), C.byref(kv), llmq.int_array(ids[5:]), 25, C.byref(llmq.host_tensor(row)))
    llmq.check(lib)
    assert kv.len == 30 and bits_equal(row[0], want[29])
    free_all(lib, m, [kv])


def test_decode_batch_8b_shapes_vs_oracle(lib, orc):
    """LLaMA-3-8B layer shapes, 2 layers, 3 sequences: the GEMMs run with
    split-K (few slabs per row block) and the SwiGLU / logits epilogues."""
    cfg = dict(vocab=128256, d_model=4096, n_layers=2, n_heads=32, n_kv=8, head_dim=128, d_ff=14336,
               max_seq=64, rope_base=500000.0, eps=1e-5)
    m = synth(lib, cfg, seed=1234)
    seqs = [[17, 128000, 42], [9, 99], [5, 6, 7, 8]]
    kvs = [new_kv(lib, m) for _ in seqs]
    for kv, s in zip(kvs, seqs):
        gpu_decode(lib, m, s[:-1], kv=kv)
    got = batch_step(lib, m, kvs, [s[-1] for s in seqs])
    for b, s in enumerate(seqs):
        want, _ = orc_decode(orc, m, s)
        assert bits_equal(got[b], want[-1]), f"sequence {b}"
    free_all(lib, m, kvs)


def test_batch_errors_leave_lengths(lib):
    m = synth(lib, dict(TINY, max_seq=4), seed=6)
    a, b = new_kv(lib, m), new_kv(lib, m)
    out = np.zeros((2, m.vocab), np.float32)
    t = llmq.host_tensor(out)
    lib.q_llama_clear_error()
    lib.q_llama_decode_batch(C.byref(m), llmq.kv_pointers([a, a]), llmq.int_array([1, 2]), 2, C.byref(t))
    assert lib.q_llama_last_error() == 1 and a.len == 0
    lib.q_llama_clear_error()
    lib.q_llama_decode_batch(C.byref(m), llmq.kv_pointers([a, b]), llmq.int_array([1, m.vocab]), 2, C.byref(t))
    assert lib.q_llama_last_error() == 1 and (a.len, b.len) == (0, 0)
    lib.q_llama_clear_error()
    lib.q_llama_prefill(C.byref(m), C.byref(a), llmq.int_array([1, 2, 3, 4, 5]), 5, None)
    assert lib.q_llama_last_error() == 1 and a.len == 0
    lib.q_llama_clear_error()
    free_all(lib, m, [a, b])
