"""CPU: pins the oracle restatement against the reference's own code (compiled
into oracle/_ref/) and against the committed golden vectors.  Bit-exact."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

import llmq
from conftest import GOLDEN
from helpers import bits_equal, bp, fp, orc_decode, orc_qmatmul, orc_quantize


def ref_quantize(ref, W):
    rows, cols = W.shape
    q = np.zeros((rows, cols), np.int8)
    s = np.zeros(cols, np.float32)
    ref.quantize_int8_percol(fp(W), rows, cols, bp(q), fp(s))
    return q, s


def ref_qmatmul(ref, A, q, s):
    out = np.zeros((A.shape[0], q.shape[1]), np.float32)
    ta, tc = llmq.host_tensor(A), llmq.host_tensor(out)
    qt = llmq.qtensor_view(q, s)
    ref.qmatmul(C.byref(ta), C.byref(qt), C.byref(tc))
    return out


def load_with(fn, path):
    m = llmq.QLlamaModel()
    assert fn(path.encode(), C.byref(m)) == 0
    return m


# ------------------------------------------------------------- golden pins
def test_golden_quant20(orc):
    d = np.load(os.path.join(GOLDEN, "quant20.npz"))
    q, s = orc_quantize(orc, d["W"])
    np.testing.assert_array_equal(q, d["q"])
    assert bits_equal(s, d["scale"])
    assert bits_equal(orc_qmatmul(orc, d["A"], q, s), d["C"])
    # the reference's own quality gate for this case (selftest.c:1205-1208)
    Wdq = (d["q"].astype(np.float32) * d["scale"][None, :]).astype(np.float32)
    Y, Yq = d["A"] @ d["W"], d["A"] @ Wdq
    assert np.sqrt(((Yq - Y) ** 2).sum() / (Y ** 2).sum()) < 0.03


def test_golden_qedge(orc):
    d = np.load(os.path.join(GOLDEN, "qedge.npz"))
    out = orc_qmatmul(orc, d["A"], d["q"], d["scale"])
    assert bits_equal(out, d["C"])
    assert np.all(out[0] == 0.0)  # an all-zero row gives exact zeros


def test_golden_selftest21(orc):
    d = np.load(os.path.join(GOLDEN, "selftest21.npz"))
    m = load_with(orc.orc_model_load, os.path.join(GOLDEN, "selftest21.llmq"))
    logits, _ = orc_decode(orc, m, d["ids"])
    assert bits_equal(logits, d["logits"])
    # the reference's own gate, int8 decode vs fp32 forward (selftest.c:1244-1246)
    f = d["fp32_logits"]
    assert np.sqrt(((logits - f) ** 2).sum() / (f ** 2).sum()) < 0.15
    orc.orc_model_free(C.byref(m))


def test_golden_mini_greedy(orc):
    d = np.load(os.path.join(GOLDEN, "mini.npz"))
    m = load_with(orc.orc_model_load, os.path.join(GOLDEN, "mini.llmq"))
    logits, _ = orc_decode(orc, m, d["fed"])
    arg = [int(orc.orc_argmax(fp(np.ascontiguousarray(r)), m.vocab)) for r in logits]
    assert arg == d["argmax"].tolist()
    assert bits_equal(logits[d["save_steps"]], d["logits"])
    orc.orc_model_free(C.byref(m))


# ------------------------------------------------- restatement vs reference
@pytest.mark.parametrize("shape", [(1, 1), (3, 5), (64, 32), (100, 37), (300, 129)])
def test_quantize_matches_reference(orc, ref, shape):
    rng = np.random.default_rng(sum(shape))
    W = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    W[:, 0] = 0.0  # an all-zero column takes scale 1
    if shape[0] > 2:
        W[1, -1] = 1e-30
    qo, so = orc_quantize(orc, W)
    qr, sr = ref_quantize(ref, W)
    np.testing.assert_array_equal(qo, qr)
    assert bits_equal(so, sr)


@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (1, 288, 96), (2, 37, 19), (5, 768, 288), (3, 4096, 64)])
def test_qmatmul_matches_reference(orc, ref, M, K, N):
    rng = np.random.default_rng(M * 1000 + K + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    q = rng.integers(-127, 128, size=(K, N)).astype(np.int8)
    s = rng.uniform(1e-3, 1e-2, size=N).astype(np.float32)
    assert bits_equal(orc_qmatmul(orc, A, q, s), ref_qmatmul(ref, A, q, s))


def test_rmsnorm_matches_reference(orc, ref):
    rng = np.random.default_rng(3)
    for n in (8, 288, 4096):
        x = (rng.standard_normal(n) * 3).astype(np.float32)
        g = rng.uniform(0.5, 1.5, n).astype(np.float32)
        y = np.zeros(n, np.float32)
        orc.orc_rmsnorm_row(fp(x), fp(g), n, 1e-5, fp(y))
        x2, yr = x[None, :].copy(), np.zeros((1, n), np.float32)
        tx, tg, ty = llmq.host_tensor(x2), llmq.host_tensor(g), llmq.host_tensor(yr)
        ref.rmsnorm(C.byref(tx), C.byref(tg), C.byref(ty), 1e-5)
        assert bits_equal(y, yr[0])


@pytest.mark.parametrize("heads,hd,base", [(6, 48, 10000.0), (32, 128, 500000.0), (4, 2, 10000.0)])
def test_rope_matches_reference(orc, ref, heads, hd, base):
    rng = np.random.default_rng(heads + hd)
    for pos in (0, 1, 7, 255, 767, 2175, 8191):
        x = rng.standard_normal(heads * hd).astype(np.float32)
        a = x.copy()
        orc.orc_rope_heads_pos_row(fp(a), heads, hd, base, pos)
        b = x[None, :].copy()
        tb = llmq.host_tensor(b)
        ref.rope_heads_pos(C.byref(tb), heads, base, pos)
        assert bits_equal(a, b[0]), pos


def test_decode_matches_reference(orc, ref):
    for name in ("selftest21", "mini"):
        path = os.path.join(GOLDEN, name + ".llmq")
        mo = load_with(orc.orc_model_load, path)
        mr = load_with(ref.q_llama_model_load, path)
        rng = np.random.default_rng(11)
        ids = rng.integers(0, mo.vocab, size=40)
        lo, _ = orc_decode(orc, mo, ids)
        kv = ref.q_llama_kv_create(C.byref(mr))
        row = np.zeros((1, mr.vocab), np.float32)
        t = llmq.host_tensor(row)
        for i, tok in enumerate(ids):
            ref.q_llama_decode_step(C.byref(mr), C.byref(kv), int(tok), C.byref(t))
            assert bits_equal(lo[i], row[0]), (name, i)
        ref.llama_kv_free(C.byref(kv))
        orc.orc_model_free(C.byref(mo))
        ref.q_llama_model_free(C.byref(mr))


def test_llmq_writer_roundtrip_through_reference_loader(orc, ref, tmp_path):
    """orc_model_save writes what the reference loader (llama.c:610-657) reads."""
    mo = load_with(orc.orc_model_load, os.path.join(GOLDEN, "mini.llmq"))
    p = str(tmp_path / "rt.llmq")
    assert orc.orc_model_save(p.encode(), C.byref(mo)) == 0
    mr = load_with(ref.q_llama_model_load, p)
    from helpers import assert_models_equal
    assert_models_equal(mo, mr)
    orc.orc_model_free(C.byref(mo))
    ref.q_llama_model_free(C.byref(mr))
