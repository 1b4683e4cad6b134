"""Small wrappers shared by the tests: run the same computation through the
oracle restatement, the reference build and libllmq_cuda.so."""
from __future__ import annotations

import ctypes as C

import numpy as np

import llmq
from llmq import c_byte_p, c_float_p, c_int_p


def fp(a: np.ndarray):
    return a.ctypes.data_as(c_float_p)


def bp(a: np.ndarray):
    return a.ctypes.data_as(c_byte_p)


# ------------------------------------------------------------------- oracle
def orc_quantize(orc, W: np.ndarray):
    rows, cols = W.shape
    q = np.zeros((rows, cols), np.int8)
    s = np.zeros(cols, np.float32)
    orc.orc_quantize_int8_percol(fp(W), rows, cols, bp(q), fp(s))
    return q, s


def orc_qmatmul(orc, A: np.ndarray, q: np.ndarray, s: np.ndarray) -> np.ndarray:
    M, K = A.shape
    N = q.shape[1]
    out = np.zeros((M, N), np.float32)
    orc.orc_qmatmul(fp(A), M, K, bp(q), fp(s), N, fp(out))
    return out


def orc_decode(orc, m, tokens, kv=None):
    """Feeds `tokens` one by one through the oracle; returns (logits rows, kv)."""
    own = kv is None
    if own:
        kv = orc.orc_kv_create(C.byref(m))
    out = np.zeros((len(tokens), m.vocab), np.float32)
    for i, t in enumerate(tokens):
        orc.orc_decode_step(C.byref(m), C.byref(kv), int(t), fp(out[i]))
    if own:
        orc.orc_kv_free(C.byref(kv))
        kv = None
    return out, kv


def orc_greedy(orc, m, prompt, n_new):
    """Prompt then n_new greedy steps; returns (fed ids, argmax per step, logits)."""
    kv = orc.orc_kv_create(C.byref(m))
    fed, arg, logits = [], [], []
    row = np.zeros(m.vocab, np.float32)
    tok = int(prompt[0])
    for step in range(len(prompt) + n_new):
        fed.append(tok)
        orc.orc_decode_step(C.byref(m), C.byref(kv), tok, fp(row))
        nxt = int(orc.orc_argmax(fp(row), m.vocab))
        arg.append(nxt)
        logits.append(row.copy())
        tok = int(prompt[step + 1]) if step + 1 < len(prompt) else nxt
    orc.orc_kv_free(C.byref(kv))
    return fed, arg, np.stack(logits)


# --------------------------------------------------------------------- gpu
def gpu_qmatmul(lib, A: np.ndarray, q: np.ndarray, s: np.ndarray) -> np.ndarray:
    M, K = A.shape
    out = np.full((M, q.shape[1]), np.nan, np.float32)
    ta, tc = llmq.host_tensor(A), llmq.host_tensor(out)
    qt = llmq.qtensor_view(q, s)
    lib.qmatmul(C.byref(ta), C.byref(qt), C.byref(tc))
    llmq.check(lib)
    return out


def gpu_quantize(lib, W: np.ndarray):
    rows, cols = W.shape
    q = np.zeros((rows, cols), np.int8)
    s = np.zeros(cols, np.float32)
    lib.quantize_int8_percol(fp(W), rows, cols, bp(q), fp(s))
    llmq.check(lib)
    return q, s


def gpu_decode(lib, m, tokens, kv=None):
    own = kv is None
    if own:
        kv = lib.q_llama_kv_create(C.byref(m))
        llmq.check(lib)
    out = np.full((len(tokens), m.vocab), np.nan, np.float32)
    row = np.zeros((1, m.vocab), np.float32)
    t = llmq.host_tensor(row)
    for i, tok in enumerate(tokens):
        lib.q_llama_decode_step(C.byref(m), C.byref(kv), int(tok), C.byref(t))
        llmq.check(lib)
        out[i] = row[0]
    if own:
        lib.llama_kv_free(C.byref(kv))
        kv = None
    return out, kv


def synth(lib, cfg: dict, seed=1234, stddev=0.02, with_bias=False):
    m = llmq.QLlamaModel()
    c = llmq.config(**cfg)
    rc = lib.llmq_synth_model(C.byref(c), seed, stddev, 1 if with_bias else 0, C.byref(m))
    assert rc == 0, lib.q_llama_last_error_message()
    return m


def model_arrays(m) -> dict:
    """Every tensor of a QLlamaModel as numpy copies (for equality checks)."""
    out = {"wte": llmq.qtensor_arrays(m.wte), "final_norm": llmq.vec_array(m.final_norm),
           "lm_head": llmq.qtensor_arrays(m.lm_head)}
    for l in range(m.n_layers):
        b = m.blocks[l]
        for n in ("attn_norm", "ffn_norm", "b_q", "b_k", "b_v"):
            out[f"{l}.{n}"] = llmq.vec_array(getattr(b, n))
        for n in ("Wq", "Wk", "Wv", "Wo", "Wgate", "Wup", "Wdown"):
            out[f"{l}.{n}"] = llmq.qtensor_arrays(getattr(b, n))
    return out


def assert_models_equal(a, b):
    da, db = model_arrays(a), model_arrays(b)
    assert da.keys() == db.keys()
    for k in da:
        x, y = da[k], db[k]
        if isinstance(x, tuple):
            np.testing.assert_array_equal(x[0], y[0], err_msg=k)
            np.testing.assert_array_equal(x[1].view(np.uint32), y[1].view(np.uint32), err_msg=k)
        else:
            np.testing.assert_array_equal(x.view(np.uint32), y.view(np.uint32), err_msg=k)


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    return a.shape == b.shape and np.array_equal(np.ascontiguousarray(a).view(np.uint32),
                                                 np.ascontiguousarray(b).view(np.uint32))


TINY = dict(vocab=32000, d_model=288, n_layers=6, n_heads=6, n_kv=2, head_dim=48, d_ff=768, max_seq=256,
            rope_base=10000.0, eps=1e-5)


# ------------------------------------------------------------------ sampler
def sampler_rows(seed=2024) -> dict:
    """Logits rows for the sampler tests: smooth, peaked, tied, flat, with NaN
    and infinities, tiny and 8B-vocabulary sized."""
    g = np.random.default_rng(seed)
    f32 = np.float32
    rows = {
        "normal32k": g.normal(0, 2, 32000).astype(f32),
        "normal128k": g.normal(0, 3, 128256).astype(f32),
        "ties": (np.round(g.normal(0, 2, 32000) * 2) / 2).astype(f32),
        "flat": np.zeros(5000, f32),
        "wide": g.normal(0, 60, 20000).astype(f32),  # most probabilities underflow to 0
        "small": g.normal(0, 1, 7).astype(f32),
        "v1024": g.normal(0, 1, 1024).astype(f32),
    }
    peaked = g.normal(0, 1, 128256).astype(f32)
    peaked[g.integers(0, 128256, 30)] += 9.0
    rows["peaked128k"] = peaked
    nan0 = g.normal(0, 1, 1000).astype(f32)
    nan0[0] = np.nan
    rows["nan_first"] = nan0
    nanm = g.normal(0, 1, 1000).astype(f32)
    nanm[500] = np.nan
    rows["nan_middle"] = nanm
    ninf = g.normal(0, 1, 2000).astype(f32)
    ninf[g.integers(0, 2000, 300)] = -np.inf
    rows["neg_inf"] = ninf
    pinf = g.normal(0, 1, 2000).astype(f32)
    pinf[77] = np.inf
    rows["pos_inf"] = pinf
    return rows


# (temperature, top_k, top_p): the CLI's settings (main.c:643-645, 771-772),
# the selftest's (selftest.c:329-337), and the edges of each knob
SAMPLER_SETTINGS = [
    (0.8, 40, 0.95), (0.9, 40, 0.95), (1.0, 1, 1.0), (0.8, 8, 0.95), (1.0, 1024, 1.0), (1.5, 1024, 0.5),
    (0.3, 40, 1.0), (1.0, 40, 0.0), (1.0, 50, 1e-9), (2.0, 700, 0.999), (0.0, 40, 0.95), (-1.0, 0, 1.0),
    (1.0, 0, 1.0), (1.0, 0, 0.9), (float("nan"), 40, 0.95),
]


def sampler_k(V: int, top_k: int) -> int:
    """Candidates the reference keeps after top-k (sampler.c:87-88)."""
    return top_k if 0 < top_k < V else V


def ref_sample(ref, row: np.ndarray, T, top_k, top_p, state: int) -> tuple[int, int]:
    t = llmq.host_tensor(row.reshape(1, -1))
    r = llmq.Rng(state)
    tok = ref.sample_token(C.byref(t), 0, T, top_k, top_p, C.byref(r))
    return tok, r.state


def orc_sample(orc, row: np.ndarray, T, top_k, top_p, state: int) -> tuple[int, int]:
    st = C.c_ulonglong(state)
    tok = orc.orc_sample_token(fp(row), row.size, T, top_k, top_p, C.byref(st))
    return tok, st.value
