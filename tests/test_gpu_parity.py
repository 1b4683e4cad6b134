"""GPU parity: libllmq_cuda.so against the oracle restatement (itself pinned to
the reference) and the golden vectors.  The bar is bit-identical output: same
int8 codes and scales, same f32 logits, same greedy ids."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

import llmq
from conftest import GOLDEN
from helpers import (TINY, bits_equal, fp, gpu_decode, gpu_qmatmul, gpu_quantize, orc_decode, orc_greedy,
                     orc_qmatmul, orc_quantize, synth)

pytestmark = pytest.mark.gpu


def load_gpu(lib, path):
    m = llmq.QLlamaModel()
    assert lib.q_llama_model_load(path.encode(), C.byref(m)) == 0, lib.q_llama_last_error_message()
    return m


# ----------------------------------------------------------- quantisation
@pytest.mark.parametrize("shape", [(1, 1), (3, 5), (64, 32), (300, 129), (4096, 1024)])
def test_quantize_bit_exact(lib, orc, shape):
    rng = np.random.default_rng(sum(shape))
    W = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    W[:, 0] = 0.0
    if shape[0] > 3:
        W[2, -1] = 1e-30
        W[3, -1] = -3e4
    qg, sg = gpu_quantize(lib, W)
    qo, so = orc_quantize(orc, W)
    np.testing.assert_array_equal(qg, qo)
    assert bits_equal(sg, so)


def test_quantize_golden_quant20(lib):
    d = np.load(os.path.join(GOLDEN, "quant20.npz"))
    q, s = gpu_quantize(lib, d["W"])
    np.testing.assert_array_equal(q, d["q"])
    assert bits_equal(s, d["scale"])


def test_dequantize_bit_exact(lib, orc):
    rng = np.random.default_rng(4)
    q = rng.integers(-127, 128, size=(70, 33)).astype(np.int8)
    s = rng.uniform(1e-3, 1e-2, 33).astype(np.float32)
    wg, wo = np.zeros((70, 33), np.float32), np.zeros((70, 33), np.float32)
    lib.dequantize_int8_percol(q.ctypes.data_as(llmq.c_byte_p), fp(s), 70, 33, fp(wg))
    llmq.check(lib)
    orc.orc_dequantize_int8_percol(q.ctypes.data_as(llmq.c_byte_p), fp(s), 70, 33, fp(wo))
    assert bits_equal(wg, wo)


# ----------------------------------------------------------------- qmatmul
@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (1, 16, 256), (2, 37, 19), (3, 100, 300), (1, 288, 32000),
                                   (8, 768, 288), (9, 64, 1000), (17, 288, 96), (1, 4096, 4096),
                                   (1, 14336, 4096), (4, 4096, 1024),
                                   # 8 rows at K = 14336: the GEMV's 16 KB tiles (KT = 64)
                                   (8, 14336, 4096), (8, 28672, 1024),
                                   # tcgen05 tensor-core path (M > 8): one and several 128-row blocks
                                   (64, 4096, 4096), (128, 4096, 1024), (200, 768, 300), (256, 4096, 4096), (64, 14336, 1024),
                                   (33, 37, 19), (64, 4096, 14336)])
def test_qmatmul_bit_exact(lib, orc, M, K, N):
    rng = np.random.default_rng(M * 7919 + K * 31 + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    q = rng.integers(-127, 128, size=(K, N)).astype(np.int8)
    s = rng.uniform(1e-3, 1e-2, size=N).astype(np.float32)
    assert bits_equal(gpu_qmatmul(lib, A, q, s), orc_qmatmul(orc, A, q, s))


def test_qmatmul_golden_edges(lib):
    for name in ("quant20", "qedge"):
        d = np.load(os.path.join(GOLDEN, name + ".npz"))
        assert bits_equal(gpu_qmatmul(lib, d["A"], d["q"], d["scale"]), d["C"]), name


def test_qmatmul_sees_weights_rewritten_in_place(lib, orc):
    """A QTensor re-quantised in place between calls is seen by the next qmatmul."""
    t = lib.qtensor_create(64, 40)
    rng = np.random.default_rng(8)
    A = rng.standard_normal((1, 64)).astype(np.float32)
    outs = []
    for seed in (1, 2):
        W = rng.standard_normal((64, 40)).astype(np.float32)
        lib.qtensor_quantize(C.byref(t), fp(W))
        llmq.check(lib)
        out = np.zeros((1, 40), np.float32)
        ta, tc = llmq.host_tensor(A), llmq.host_tensor(out)
        lib.qmatmul(C.byref(ta), C.byref(t), C.byref(tc))
        llmq.check(lib)
        q, s = llmq.qtensor_arrays(t)
        assert bits_equal(out, orc_qmatmul(orc, A, q, s))
        outs.append(out)
    assert not np.array_equal(outs[0], outs[1])
    lib.qtensor_free(C.byref(t))


# ------------------------------------------------------------------ decode
def test_decode_golden_selftest21(lib):
    d = np.load(os.path.join(GOLDEN, "selftest21.npz"))
    m = load_gpu(lib, os.path.join(GOLDEN, "selftest21.llmq"))
    logits, _ = gpu_decode(lib, m, d["ids"])
    assert bits_equal(logits, d["logits"])
    lib.q_llama_model_free(C.byref(m))


def test_decode_golden_mini_300_steps(lib):
    """Biases, rope_base 5e5, positions 0..299: identical logits and ids."""
    d = np.load(os.path.join(GOLDEN, "mini.npz"))
    m = load_gpu(lib, os.path.join(GOLDEN, "mini.llmq"))
    logits, _ = gpu_decode(lib, m, d["fed"])
    assert bits_equal(logits[d["save_steps"]], d["logits"])
    arg = logits.argmax(axis=1)  # numpy argmax also returns the first maximum
    assert arg.tolist() == d["argmax"].tolist()
    lib.q_llama_model_free(C.byref(m))


def test_decode_tiny_config_vs_oracle(lib, orc):
    """configs[0] shape (dm 288, 6 layers, GQA 6/2, hd 48, vocab 32000)."""
    m = synth(lib, TINY, seed=1234, with_bias=True)
    rng = np.random.default_rng(5678)
    prompt = rng.integers(0, TINY["vocab"], 16)
    fed, arg, ologits = orc_greedy(orc, m, prompt, 24)
    glogits, _ = gpu_decode(lib, m, fed)
    assert bits_equal(glogits, ologits)
    assert glogits.argmax(axis=1).tolist() == arg
    lib.q_llama_model_free(C.byref(m))


def test_decode_8b_shapes_two_layers_vs_oracle(lib, orc):
    """LLaMA-3-8B layer and head shapes (dm 4096, GQA 32/8, hd 128, dff 14336,
    vocab 128256, rope 5e5) with 2 layers, so the CPU oracle stays fast."""
    cfg = dict(vocab=128256, d_model=4096, n_layers=2, n_heads=32, n_kv=8, head_dim=128, d_ff=14336,
               max_seq=64, rope_base=500000.0, eps=1e-5)
    m = synth(lib, cfg, seed=1234)
    ids = [17, 128000, 42, 9999]
    ologits, _ = orc_decode(orc, m, ids)
    glogits, _ = gpu_decode(lib, m, ids)
    assert bits_equal(glogits, ologits)
    lib.q_llama_model_free(C.byref(m))


def test_70b_shapes_two_layers_vs_oracle(lib, orc):
    """LLaMA-3-70B layer and head shapes (dm 8192, GQA 64/8, hd 128, dff 28672,
    vocab 128256, rope 5e5) with 2 layers: the 8192-term RMSNorm chains, the
    28672-deep W2 product and the 8-head query groups.  Single-sequence steps,
    a prefill and a 3-row batched step, all against the oracle's sequential
    decode, bit for bit."""
    cfg = dict(vocab=128256, d_model=8192, n_layers=2, n_heads=64, n_kv=8, head_dim=128, d_ff=28672,
               max_seq=32, rope_base=500000.0, eps=1e-5)
    m = synth(lib, cfg, seed=4321)
    ids = [17, 128000, 42, 9999, 5]
    # oracle: the five ids, then one more step of token 77 on the same cache
    okv = orc.orc_kv_create(C.byref(m))
    want = np.zeros((len(ids) + 1, cfg["vocab"]), np.float32)
    for i, tok in enumerate(ids + [77]):
        orc.orc_decode_step(C.byref(m), C.byref(okv), int(tok), fp(want[i]))
    orc.orc_kv_free(C.byref(okv))
    # single-sequence steps
    kv1 = lib.q_llama_kv_create(C.byref(m))
    got, _ = gpu_decode(lib, m, ids, kv=kv1)
    assert bits_equal(got, want[:len(ids)])
    # a prefill of the first four ids (logits of the last row)
    kv2 = lib.q_llama_kv_create(C.byref(m))
    row = np.zeros((1, cfg["vocab"]), np.float32)
    t = llmq.host_tensor(row)
    lib.q_llama_prefill(C.byref(m), C.byref(kv2), llmq.int_array(ids[:4]), 4, C.byref(t))
    llmq.check(lib)
    assert bits_equal(row[0], want[3])
    # one batched step of three sequences at positions 5, 4 and 0
    kv3 = lib.q_llama_kv_create(C.byref(m))
    out = np.zeros((3, cfg["vocab"]), np.float32)
    to = llmq.host_tensor(out)
    lib.q_llama_decode_batch(C.byref(m), llmq.kv_pointers([kv1, kv2, kv3]), llmq.int_array([77, ids[4], ids[0]]), 3,
                             C.byref(to))
    llmq.check(lib)
    assert bits_equal(out[0], want[5]) and bits_equal(out[1], want[4]) and bits_equal(out[2], want[0])
    assert (kv1.len, kv2.len, kv3.len) == (6, 5, 1)
    for kv in (kv1, kv2, kv3):
        lib.llama_kv_free(C.byref(kv))
    lib.q_llama_model_free(C.byref(m))


def test_decode_long_cache_vs_oracle(lib, orc):
    """max_seq 2048: the softmax-V kernel streams the value rows through its
    ring (shorter caches stage the whole value slice at once)."""
    m = synth(lib, dict(TINY, max_seq=2048), seed=31, with_bias=True)
    ids = np.random.default_rng(2).integers(0, TINY["vocab"], 140).tolist()
    ologits, _ = orc_decode(orc, m, ids)
    glogits, _ = gpu_decode(lib, m, ids)
    assert bits_equal(glogits, ologits)
    lib.q_llama_model_free(C.byref(m))


def test_attention_path_choice(lib):
    """The fused cluster attention is taken wherever its shared memory fits
    (the 8B headline cache, a 1400-position cache with 32-row key chunks); the
    two-kernel path beyond (TINY heads at max_seq 2048, covered above)."""
    assert lib.llmq_attention_launches(32, 8, 128, 768) == 1
    assert lib.llmq_attention_launches(4, 2, 128, 1400) == 1
    assert lib.llmq_attention_launches(TINY["n_heads"], TINY["n_kv"], TINY["head_dim"], 2048) == 2


def test_decode_fused_attention_key_chunks_vs_oracle(lib, orc):
    """hd 128 at max_seq 1400: a part of the positions does not fit in shared
    memory at once, so the fused kernel streams its keys through two slots;
    300 positions, GQA 4/2."""
    cfg = dict(vocab=512, d_model=256, n_layers=2, n_heads=4, n_kv=2, head_dim=128, d_ff=512, max_seq=1400,
               rope_base=10000.0, eps=1e-5)
    m = synth(lib, cfg, seed=41, with_bias=True)
    ids = np.random.default_rng(4).integers(0, cfg["vocab"], 300).tolist()
    ologits, _ = orc_decode(orc, m, ids)
    glogits, _ = gpu_decode(lib, m, ids)
    assert bits_equal(glogits, ologits)
    lib.q_llama_model_free(C.byref(m))


def test_generate_matches_stepwise_argmax(lib):
    m = synth(lib, TINY, seed=77)
    kv1 = lib.q_llama_kv_create(C.byref(m))
    ids = (C.c_int * 30)()
    assert lib.q_llama_generate(C.byref(m), C.byref(kv1), 5, 30, ids) == 0
    assert kv1.len == 30
    kv2 = lib.q_llama_kv_create(C.byref(m))
    tok, seq = 5, []
    for _ in range(30):
        tok = lib.q_llama_decode_step_argmax(C.byref(m), C.byref(kv2), tok, None)
        seq.append(tok)
    llmq.check(lib)
    assert list(ids) == seq
    lib.llama_kv_free(C.byref(kv1))
    lib.llama_kv_free(C.byref(kv2))
    lib.q_llama_model_free(C.byref(m))


def test_kv_sync_host_matches_oracle_cache(lib, orc):
    m = synth(lib, TINY, seed=3)
    ids = [1, 2, 3, 4, 5, 6, 7]
    _, okv = orc_decode(orc, m, ids, kv=orc.orc_kv_create(C.byref(m)))
    gkv = lib.q_llama_kv_create(C.byref(m))
    gpu_decode(lib, m, ids, kv=gkv)
    assert lib.q_llama_kv_sync_host(C.byref(m), C.byref(gkv)) == 0
    n = len(ids) * gkv.kv_dim
    for l in range(m.n_layers):
        for a, b in ((gkv.k, okv.k), (gkv.v, okv.v)):
            x = np.ctypeslib.as_array(a[l], shape=(n,))
            y = np.ctypeslib.as_array(b[l], shape=(n,))
            assert bits_equal(x, y)
    orc.orc_kv_free(C.byref(okv))
    lib.llama_kv_free(C.byref(gkv))
    lib.q_llama_model_free(C.byref(m))


def test_continues_a_cache_filled_by_the_reference(lib, ref):
    """A LlamaKV whose first positions were decoded by the reference CPU code is
    adopted by the GPU path, which continues bit-identically."""
    m = load_gpu(lib, os.path.join(GOLDEN, "mini.llmq"))
    d = np.load(os.path.join(GOLDEN, "mini.npz"))
    kv = ref.q_llama_kv_create(C.byref(m))
    row = np.zeros((1, m.vocab), np.float32)
    t = llmq.host_tensor(row)
    fed = d["fed"]
    for tok in fed[:20]:
        ref.q_llama_decode_step(C.byref(m), C.byref(kv), int(tok), C.byref(t))
    glogits, _ = gpu_decode(lib, m, fed[20:120], kv=kv)
    assert glogits.argmax(axis=1).tolist() == d["argmax"][20:120].tolist()
    assert bits_equal(glogits[100 - 20], d["logits"][list(d["save_steps"]).index(100)])
    ref.llama_kv_free(C.byref(kv))
    lib.q_llama_model_free(C.byref(m))


def test_bad_token_and_full_cache_are_errors(lib):
    m = synth(lib, dict(TINY, max_seq=4), seed=5)
    kv = lib.q_llama_kv_create(C.byref(m))
    row = np.zeros((1, m.vocab), np.float32)
    t = llmq.host_tensor(row)
    lib.q_llama_clear_error()
    lib.q_llama_decode_step(C.byref(m), C.byref(kv), m.vocab, C.byref(t))
    assert lib.q_llama_last_error() == 1 and kv.len == 0
    lib.q_llama_clear_error()
    for i in range(4):
        lib.q_llama_decode_step(C.byref(m), C.byref(kv), i, C.byref(t))
        llmq.check(lib)
    lib.q_llama_decode_step(C.byref(m), C.byref(kv), 0, C.byref(t))
    assert lib.q_llama_last_error() == 1 and kv.len == 4
    lib.q_llama_clear_error()
    lib.llama_kv_free(C.byref(kv))
    lib.q_llama_model_free(C.byref(m))


# -------------------------------------------------------------------- expf
def test_device_expf_equals_host_libm_on_every_float(lib, orc):
    """The device expf used by softmax and SiLU returns the host C library's
    expf bit for bit on all 2^32 inputs (NaN inputs: both NaN)."""
    chunk = 1 << 26
    dev = np.empty(chunk, np.float32)
    host = np.empty(chunk, np.float32)
    mismatches = 0
    for first in range(0, 1 << 32, chunk):
        x = np.arange(first, first + chunk, dtype=np.uint64).astype(np.uint32).view(np.float32)
        assert lib.llmq_expf_device(fp(x), fp(dev), chunk) == 0
        orc.orc_expf_bits(first, chunk, fp(host))
        same = dev.view(np.uint32) == host.view(np.uint32)
        same |= np.isnan(dev) & np.isnan(host)
        mismatches += int((~same).sum())
    assert mismatches == 0


# ----------------------------------------- RMSNorm prologue on rounding ties
def _emulated_code_flips(x, g, eps=np.float32(1e-5)):
    """How many activation codes differ between the exact scale (the
    sequential f32 sum of squares, rmsnorm.c:15) and a scale from the
    double-precision sum of the same squares: how sensitive the row is to the
    order of that sum."""
    f32 = np.float32

    def r_of(ms):
        ms = f32(ms * f32(f32(1) / f32(len(x))))
        return f32(f32(1) / np.sqrt(f32(ms + eps)))

    def codes(r):
        y = ((x * r).astype(f32) * g).astype(f32)
        a = f32(np.max(np.abs(y)) / f32(127))
        return np.clip(np.rint((y * f32(f32(1) / a)).astype(f32)), -127, 127)

    sq = (x * x).astype(f32)
    ms = f32(0)
    for v in sq:
        ms = f32(ms + v)
    return int(np.sum(codes(r_of(ms)) != codes(r_of(f32(np.sum(sq.astype(np.float64)))))))


@pytest.mark.parametrize("ties", [4095, 60, 20, 0])
def test_rmsnorm_gemv_on_rounding_ties(lib, orc, ties):
    """Rows whose normalised values sit at .5 rounding ties, so that any
    deviation from the reference's sequential sum of squares would flip codes:
    with the scale from an exactly rounded sum, 560, 47 and 4 of the codes
    differ; and a plain row.  The GEMV with the RMSNorm prologue must equal
    rmsnorm + qmatmul of the oracle bit for bit."""
    f32 = np.float32
    rng = np.random.default_rng(7 + ties)
    K, N = 4096, 1000
    x = (rng.standard_normal(K) * 10).astype(f32)
    if ties:
        x[1:1 + ties] = ((rng.integers(-126, 126, ties) + 0.5) * 100.0 / 127).astype(f32)
        x[0] = f32(100.0)
    g = np.ones(K, f32) if ties else rng.uniform(0.5, 1.5, K).astype(f32)
    flips = _emulated_code_flips(x, g)
    if ties == 4095:
        assert flips > 256
    elif ties:
        assert 0 < flips <= 256
    q = rng.integers(-127, 128, size=(K, N)).astype(np.int8)
    s = rng.uniform(1e-3, 1e-2, size=N).astype(f32)
    y = np.zeros(K, f32)
    orc.orc_rmsnorm_row(fp(x), fp(g), K, f32(1e-5), fp(y))
    want = orc_qmatmul(orc, y.reshape(1, K), q, s)[0]
    got = np.full(N, np.nan, f32)
    qt = llmq.qtensor_view(q, s)
    assert lib.llmq_rmsnorm_qmatmul(fp(x), fp(g), f32(1e-5), C.byref(qt), fp(got)) == 0, \
        lib.q_llama_last_error_message()
    assert bits_equal(got, want)


def test_measurement_hooks_run(lib):
    """The timing entry points bench.py reads (per-kind GEMV and attention
    timings from a captured graph, the per-kernel step profile, the isolated
    product) run and report positive times."""
    m = synth(lib, dict(TINY, n_layers=3), seed=9)
    kv = lib.q_llama_kv_create(C.byref(m))
    gpu_decode(lib, m, [1, 2, 3], kv=kv)
    for which in range(6):
        ms, by = C.c_float(), C.c_double()
        assert lib.llmq_bench_gemv(C.byref(m), which, 1, 5, C.byref(ms), C.byref(by)) == 0, \
            lib.q_llama_last_error_message()
        assert ms.value > 0 and by.value > 0, which
    nk = lib.llmq_kernels_per_step(C.byref(m))
    prof = np.zeros(nk, np.float32)
    assert lib.llmq_step_profile(C.byref(m), C.byref(kv), 4, prof.ctypes.data_as(llmq.c_float_p), nk) == 0
    assert kv.len == 4 and np.all(prof > 0)
    t = lib.qtensor_create(288, 768)
    lib.llmq_synth_qtensor(C.byref(t), 5)
    for M in (1, 3, 64):
        ms = C.c_float()
        assert lib.llmq_bench_qmatmul(C.byref(t), M, 3, C.byref(ms)) == 0 and ms.value > 0
    lib.qtensor_free(C.byref(t))
    lib.llama_kv_free(C.byref(kv))
    lib.q_llama_model_free(C.byref(m))
