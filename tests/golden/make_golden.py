"""Regenerates the golden fixtures in this directory from the reference itself.

Runs the reference's own C code (compiled from its sources into oracle/_ref/ by
oracle/Makefile) on:
  * quant20.npz  - selftest part [20]'s inputs (selftest.c:1186-1192):
                   quantize_int8_percol codes/scales and qmatmul of A with them
  * qedge.npz    - qmatmul edge rows: all-zero row, exact .5 ties, a lone
                   large value, tiny values; K=37 and N=19 (not tile multiples)
  * selftest21.* - selftest part [21]'s model (selftest.c:1221-1230: srand(17),
                   llama_model_randomize, q_llama_quantize_from), saved as LLMQ,
                   plus its int8 decode logits for ids {3,7,1,9,2,5} and the fp32
                   forward logits
  * mini.*       - a larger randomised model (non-zero biases, rope_base 5e5)
                   decoded greedily from a 16-id prompt to position 300: every
                   argmax id, and the logits at selected steps
Usage: python tests/golden/make_golden.py
(needs oracle/_ref/ built from the reference sources: make -C oracle REF=<reference checkout>)
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402
import llmq  # noqa: E402

MINI_CFG = dict(vocab=512, d_model=64, n_layers=2, n_heads=4, n_kv=2, head_dim=16, d_ff=160, max_seq=320,
                rope_base=500000.0, eps=1e-5)
MINI_STEPS = 300
MINI_SAVE = (0, 1, 15, 16, 17, 100, 200, 299)


def quant20(ref):
    n, rows, cols = 4, 64, 32
    A = np.array([((i * 13 % 100) / 50.0) - 1.0 for i in range(n * rows)], dtype=np.float32).reshape(n, rows)
    W = np.array([((i * 29 % 100) / 50.0 - 1.0) * 0.3 for i in range(rows * cols)],
                 dtype=np.float32).reshape(rows, cols)
    q = np.zeros((rows, cols), np.int8)
    s = np.zeros(cols, np.float32)
    ref.quantize_int8_percol(W.ctypes.data_as(llmq.c_float_p), rows, cols, q.ctypes.data_as(llmq.c_byte_p),
                             s.ctypes.data_as(llmq.c_float_p))
    Cm = np.zeros((n, cols), np.float32)
    ta, tc = llmq.host_tensor(A), llmq.host_tensor(Cm)
    qt = llmq.qtensor_view(q, s)
    ref.qmatmul(C.byref(ta), C.byref(qt), C.byref(tc))
    np.savez(os.path.join(HERE, "quant20.npz"), A=A, W=W, q=q, scale=s, C=Cm)


def qedge(ref):
    rng = np.random.default_rng(7)
    K, N = 37, 19
    A = np.zeros((5, K), np.float32)
    A[1, :8] = [127.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5]  # scale 1: exact ties
    A[2, 5] = 3.0e4
    A[2, 6:] = rng.standard_normal(K - 6).astype(np.float32) * 1e-3
    A[3] = rng.standard_normal(K).astype(np.float32)
    A[4] = rng.standard_normal(K).astype(np.float32) * 1e-30
    q = rng.integers(-127, 128, size=(K, N)).astype(np.int8)
    s = rng.uniform(1e-3, 1e-2, size=N).astype(np.float32)
    Cm = np.zeros((5, N), np.float32)
    ta, tc = llmq.host_tensor(A), llmq.host_tensor(Cm)
    qt = llmq.qtensor_view(q, s)
    ref.qmatmul(C.byref(ta), C.byref(qt), C.byref(tc))
    np.savez(os.path.join(HERE, "qedge.npz"), A=A, q=q, scale=s, C=Cm)


def decode_ref(ref, qm, ids):
    kv = ref.q_llama_kv_create(C.byref(qm))
    out = []
    logits = np.zeros((1, qm.vocab), np.float32)
    lt = llmq.host_tensor(logits)
    for t in ids:
        ref.q_llama_decode_step(C.byref(qm), C.byref(kv), int(t), C.byref(lt))
        out.append(logits[0].copy())
    ref.llama_kv_free(C.byref(kv))
    return np.stack(out)


def selftest21(ref, orc):
    libc = oracle.libc()
    libc.srand(17)
    fm = ref.llama_model_create(32, 8, 2, 4, 2, 2, 16, 64, 10000.0, 1e-5)
    ref.llama_model_randomize(C.byref(fm))
    ids = np.array([3, 7, 1, 9, 2, 5], np.int32)
    lf = np.zeros((6, 32), np.float32)
    tf = llmq.host_tensor(lf)
    ref.llama_model_forward(C.byref(fm), ids.ctypes.data_as(llmq.c_int_p), 6, C.byref(tf))
    qm = ref.q_llama_quantize_from(C.byref(fm))
    path = os.path.join(HERE, "selftest21.llmq")
    assert orc.orc_model_save(path.encode(), C.byref(qm)) == 0
    logits = decode_ref(ref, qm, ids)
    np.savez(os.path.join(HERE, "selftest21.npz"), ids=ids, logits=logits, fp32_logits=lf)
    ref.q_llama_model_free(C.byref(qm))
    ref.llama_model_free(C.byref(fm))


def mini(ref, orc):
    libc = oracle.libc()
    libc.srand(2024)
    c = MINI_CFG
    fm = ref.llama_model_create(c["vocab"], c["d_model"], c["n_layers"], c["n_heads"], c["n_kv"], c["head_dim"],
                                c["d_ff"], c["max_seq"], c["rope_base"], c["eps"])
    ref.llama_model_randomize(C.byref(fm))
    qm = ref.q_llama_quantize_from(C.byref(fm))
    path = os.path.join(HERE, "mini.llmq")
    assert orc.orc_model_save(path.encode(), C.byref(qm)) == 0
    rng = np.random.default_rng(5678)
    prompt = rng.integers(0, c["vocab"], size=16).astype(np.int32)
    kv = ref.q_llama_kv_create(C.byref(qm))
    logits = np.zeros((1, c["vocab"]), np.float32)
    lt = llmq.host_tensor(logits)
    fed, argmax, saved = [], [], []
    tok = int(prompt[0])
    for step in range(MINI_STEPS):
        fed.append(tok)
        ref.q_llama_decode_step(C.byref(qm), C.byref(kv), tok, C.byref(lt))
        nxt = int(ref.sample_argmax(C.byref(lt), 0))
        argmax.append(nxt)
        if step in MINI_SAVE:
            saved.append(logits[0].copy())
        tok = int(prompt[step + 1]) if step + 1 < len(prompt) else nxt
    ref.llama_kv_free(C.byref(kv))
    np.savez(os.path.join(HERE, "mini.npz"), prompt=prompt, fed=np.array(fed, np.int32),
             argmax=np.array(argmax, np.int32), save_steps=np.array(MINI_SAVE, np.int32),
             logits=np.stack(saved))
    ref.q_llama_model_free(C.byref(qm))
    ref.llama_model_free(C.byref(fm))


def main():
    ref = oracle.load_reference()
    if ref is None:
        sys.exit("reference not built: make -C oracle (needs the reference sources)")
    orc = oracle.load_oracle()
    quant20(ref)
    qedge(ref)
    selftest21(ref, orc)
    mini(ref, orc)
    for f in sorted(os.listdir(HERE)):
        if f.endswith((".npz", ".llmq")):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
