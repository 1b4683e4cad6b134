"""The fp32 (LLMA) decode path (llama.c:296-362): the oracle restatement
pinned against the reference build on the CPU, the checkpoint reader and the
synthetic fp32 model on the CPU, then llama_decode_step on the GPU against
the oracle and against the reference itself, bit for bit."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

import llmq
from conftest import GOLDEN
from helpers import TINY, bits_equal, fp, orc_sample

F32_TINY = dict(TINY, max_seq=64)
# chain lengths that are not multiples of 4 or 8 (d_model 50, q width 50, d_ff 71)
ODD_F32 = dict(vocab=1001, d_model=50, n_layers=2, n_heads=5, n_kv=1, head_dim=10, d_ff=71, max_seq=16,
               rope_base=10000.0, eps=1e-5)


def synth_f32(lib, cfg, seed=1234, with_bias=True, stddev=0.02):
    m = llmq.LlamaModel()
    c = llmq.config(**cfg)
    assert lib.llmq_synth_model_f32(C.byref(c), seed, stddev, 1 if with_bias else 0, C.byref(m)) == 0, \
        lib.q_llama_last_error_message()
    return m


def f32_arrays(m) -> dict:
    def arr(t, n=None):
        size = t.size
        return np.ctypeslib.as_array(t.data, shape=(size,)).copy()
    out = {"wte": arr(m.wte), "final_norm": arr(m.final_norm), "lm_head": arr(m.lm_head)}
    for l in range(m.n_layers):
        b = m.blocks[l]
        for n in ("attn_norm", "ffn_norm", "b_q", "b_k", "b_v", "Wq", "Wk", "Wv", "Wo", "Wgate", "Wup", "Wdown"):
            out[f"{l}.{n}"] = arr(getattr(b, n))
    return out


def orc_f32_decode(orc, m, tokens):
    kv = orc.orc_f32_kv_create(C.byref(m))
    out = np.zeros((len(tokens), m.vocab), np.float32)
    for i, t in enumerate(tokens):
        orc.orc_f32_decode_step(C.byref(m), C.byref(kv), int(t), fp(out[i]))
    orc.orc_kv_free(C.byref(kv))
    return out


def ref_f32_decode(ref, m, tokens):
    kv = ref.llama_kv_create(C.byref(m))
    out = np.zeros((len(tokens), m.vocab), np.float32)
    row = np.zeros((1, m.vocab), np.float32)
    t = llmq.host_tensor(row)
    for i, tok in enumerate(tokens):
        ref.llama_decode_step(C.byref(m), C.byref(kv), int(tok), C.byref(t))
        out[i] = row[0]
    ref.llama_kv_free(C.byref(kv))
    return out


# ---------------------------------------------------------------- CPU only
def test_oracle_f32_decode_matches_reference(lib, orc, ref):
    """orc_f32_decode_step against the reference's llama_decode_step: a model
    with the reference's own random init, and a synthetic one with biases."""
    rm = ref.llama_model_create(512, 64, 2, 4, 2, 16, 160, 32, 10000.0, 1e-5)
    ref.llama_model_randomize(C.byref(rm))
    ids = [3, 141, 59, 26, 5, 358, 97]
    assert bits_equal(orc_f32_decode(orc, rm, ids), ref_f32_decode(ref, rm, ids))
    ref.llama_model_free(C.byref(rm))
    m = synth_f32(lib, dict(F32_TINY, n_layers=2), seed=7)
    ids = [5, 77, 31999, 0, 1234]
    assert bits_equal(orc_f32_decode(orc, m, ids), ref_f32_decode(ref, m, ids))
    lib.llmq_llama_model_free(C.byref(m))
    # the odd shapes of the GPU test (chains of 50 and 71 terms)
    m = synth_f32(lib, ODD_F32, seed=77)
    ids = [0, 1000, 5, 77, 3, 999]
    assert bits_equal(orc_f32_decode(orc, m, ids), ref_f32_decode(ref, m, ids))
    lib.llmq_llama_model_free(C.byref(m))


def test_synth_f32_is_the_dequantised_int8_model(lib):
    """llmq_synth_model_f32 = the int8 synthetic model dequantised as
    llama_model_load does for an LLMQ file (quant.c:29-33)."""
    cfg = dict(F32_TINY, n_layers=2)
    m = synth_f32(lib, cfg, seed=11)
    q = llmq.QLlamaModel()
    c = llmq.config(**cfg)
    assert lib.llmq_synth_model(C.byref(c), 11, 0.02, 1, C.byref(q)) == 0
    fa = f32_arrays(m)
    for name, qt in [("wte", q.wte), ("lm_head", q.lm_head), ("0.Wq", q.blocks[0].Wq), ("1.Wdown", q.blocks[1].Wdown)]:
        codes, scale = llmq.qtensor_arrays(qt)
        want = (codes.astype(np.float32) * scale[None, :]).astype(np.float32).ravel()
        assert np.array_equal(fa[name].view(np.uint32), want.view(np.uint32)), name
    assert np.array_equal(fa["0.b_q"], llmq.vec_array(q.blocks[0].b_q))
    lib.q_llama_model_free(C.byref(q))
    lib.llmq_llama_model_free(C.byref(m))


def test_f32_loader_matches_reference_loader(lib, ref):
    """llmq_llama_model_load of an LLMQ checkpoint = the reference's
    llama_model_load (every 2-D tensor dequantised), tensor for tensor."""
    path = os.path.join(GOLDEN, "mini.llmq").encode()
    a, b = llmq.LlamaModel(), llmq.LlamaModel()
    assert lib.llmq_llama_model_load(path, C.byref(a)) == 0
    assert ref.llama_model_load(path, C.byref(b)) == 0
    fa, fb = f32_arrays(a), f32_arrays(b)
    assert fa.keys() == fb.keys()
    for k in fa:
        assert np.array_equal(fa[k].view(np.uint32), fb[k].view(np.uint32)), k
    lib.llmq_llama_model_free(C.byref(a))
    ref.llama_model_free(C.byref(b))


def test_f32_loader_rejects_bad_files(lib, tmp_path):
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"XXXX" + b"\0" * 60)
    m = llmq.LlamaModel()
    assert lib.llmq_llama_model_load(str(bad).encode(), C.byref(m)) == 1
    assert lib.llmq_llama_model_load(str(tmp_path / "missing.bin").encode(), C.byref(m)) == 1


# --------------------------------------------------------------------- GPU
def gpu_f32_decode(lib, m, tokens):
    kv = lib.llama_kv_create(C.byref(m))
    llmq.check(lib)
    out = np.full((len(tokens), m.vocab), np.nan, np.float32)
    row = np.zeros((1, m.vocab), np.float32)
    t = llmq.host_tensor(row)
    for i, tok in enumerate(tokens):
        lib.llama_decode_step(C.byref(m), C.byref(kv), int(tok), C.byref(t))
        llmq.check(lib)
        out[i] = row[0]
    lib.llama_kv_free(C.byref(kv))
    return out


@pytest.mark.gpu
def test_f32_decode_tiny_matches_oracle(lib, orc):
    m = synth_f32(lib, F32_TINY, seed=1234)
    ids = np.random.default_rng(3).integers(0, F32_TINY["vocab"], 24).tolist()
    assert bits_equal(gpu_f32_decode(lib, m, ids), orc_f32_decode(orc, m, ids))
    lib.llmq_llama_model_free(C.byref(m))


@pytest.mark.gpu
def test_f32_decode_odd_shapes_matches_oracle(lib, orc):
    """Chain lengths that are not multiples of 4 or 8 (d_model 50, q width
    50, d_ff 71): the short tails of the tile rows and of the input rows."""
    m = synth_f32(lib, ODD_F32, seed=77)
    ids = [0, 1000, 5, 77, 3, 999]
    assert bits_equal(gpu_f32_decode(lib, m, ids), orc_f32_decode(orc, m, ids))
    lib.llmq_llama_model_free(C.byref(m))


@pytest.mark.gpu
def test_f32_decode_8b_shapes_two_layers(lib, orc):
    """LLaMA-3-8B layer shapes in fp32 (dm 4096, dff 14336: the down
    projection's chains are 14336 long; vocab 128256: 109 units per CTA)."""
    cfg = dict(vocab=128256, d_model=4096, n_layers=2, n_heads=32, n_kv=8, head_dim=128, d_ff=14336,
               max_seq=32, rope_base=500000.0, eps=1e-5)
    m = synth_f32(lib, cfg, seed=99, with_bias=False)
    ids = [17, 128000, 42]
    assert bits_equal(gpu_f32_decode(lib, m, ids), orc_f32_decode(orc, m, ids))
    lib.llmq_llama_model_free(C.byref(m))


@pytest.mark.gpu
def test_f32_checkpoint_decode_matches_reference(lib, ref):
    """An LLMQ checkpoint read as an fp32 model (llmq_llama_model_load) and
    decoded on the GPU equals the reference's llama_model_load +
    llama_decode_step."""
    path = os.path.join(GOLDEN, "mini.llmq").encode()
    a, b = llmq.LlamaModel(), llmq.LlamaModel()
    assert lib.llmq_llama_model_load(path, C.byref(a)) == 0
    assert ref.llama_model_load(path, C.byref(b)) == 0
    ids = [3, 141, 59, 26, 5, 358, 97, 93, 1, 2, 3]
    assert bits_equal(gpu_f32_decode(lib, a, ids), ref_f32_decode(ref, b, ids))
    lib.llmq_llama_model_free(C.byref(a))
    ref.llama_model_free(C.byref(b))


@pytest.mark.gpu
def test_f32_generate_and_sample(lib, orc):
    m = synth_f32(lib, F32_TINY, seed=5)
    n = 20
    # greedy: generate equals stepwise argmax
    kv = lib.llama_kv_create(C.byref(m))
    ids = (C.c_int * n)()
    assert lib.llama_generate(C.byref(m), C.byref(kv), 9, n, ids) == 0 and kv.len == n
    kv2 = lib.llama_kv_create(C.byref(m))
    tok, seq = 9, []
    for _ in range(n):
        tok = lib.llama_decode_step_argmax(C.byref(m), C.byref(kv2), tok, None)
        seq.append(tok)
    assert list(ids) == seq
    # sampled: the reference loop over the oracle
    okv = orc.orc_f32_kv_create(C.byref(m))
    row = np.zeros(m.vocab, np.float32)
    st, tok, want = lib.rng_create(1234).state, 9, []
    for _ in range(n):
        orc.orc_f32_decode_step(C.byref(m), C.byref(okv), tok, fp(row))
        tok, st = orc_sample(orc, row, 0.8, 40, 0.95, st)
        want.append(tok)
    orc.orc_kv_free(C.byref(okv))
    kv3 = lib.llama_kv_create(C.byref(m))
    r = lib.rng_create(1234)
    out = (C.c_int * n)()
    assert lib.llama_generate_sample(C.byref(m), C.byref(kv3), 9, n, 0.8, 40, 0.95, C.byref(r), out) == 0
    assert list(out) == want and r.state == st
    for k in (kv, kv2, kv3):
        lib.llama_kv_free(C.byref(k))
    lib.llmq_llama_model_free(C.byref(m))
