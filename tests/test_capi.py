"""CPU: the C-ABI library loads, exports every entry point include/llmq_cuda.h
declares, and its host-only logic (LLMQ I/O, argument checks, the synthetic
generator) behaves like the reference.  No GPU compute is called here."""
from __future__ import annotations

import ctypes as C
import os
import re
import struct
import subprocess
import sys

import numpy as np
import pytest

import llmq
from conftest import GOLDEN, ROOT, has_gpu
from helpers import assert_models_equal, synth


def declared_functions() -> list[str]:
    src = open(os.path.join(ROOT, "include", "llmq_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w \*]*?\b([a-z_][a-z0-9_]*)\s*\(", src, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "while", "sizeof")))


def test_header_declares_reference_api():
    names = declared_functions()
    for n in ("quantize_int8_percol", "dequantize_int8_percol", "qtensor_create", "qtensor_free",
              "qtensor_quantize", "qmatmul", "q_llama_model_load", "q_llama_model_free",
              "q_llama_quantize_from", "q_llama_kv_create", "llama_kv_free", "q_llama_decode_step"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", llmq.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    declared = set(declared_functions())
    assert declared <= exported, declared - exported
    assert exported <= declared, exported - declared  # nothing undeclared leaks out
    for n in declared:
        assert hasattr(lib, n)


def test_binding_covers_every_symbol():
    assert set(declared_functions()) == set(llmq.SIGNATURES)


def test_loader_rejects_bad_files(lib, tmp_path):
    good = open(os.path.join(GOLDEN, "mini.llmq"), "rb").read()
    cases = {
        "missing": None,
        "short_header": good[:20],
        "bad_magic": b"LLMA" + good[4:],
        "bad_version": good[:4] + struct.pack("<I", 1) + good[8:],
        "bad_config": good[:8] + struct.pack("<i", 0) + good[12:],
        "gqa_not_dividing": good[:20] + struct.pack("<i", 3) + good[24:],
        "truncated_weights": good[:-100],
    }
    for name, blob in cases.items():
        p = tmp_path / (name + ".llmq")
        if blob is not None:
            p.write_bytes(blob)
        m = llmq.QLlamaModel()
        assert lib.q_llama_model_load(str(p).encode(), C.byref(m)) == 1, name
    lib.q_llama_clear_error()


def test_qmatmul_rejects_bad_shapes(lib):
    A = np.zeros((2, 5), np.float32)
    out = np.zeros((2, 3), np.float32)
    q = np.zeros((4, 3), np.int8)  # K mismatch: A has 5 columns
    s = np.ones(3, np.float32)
    ta, tc = llmq.host_tensor(A), llmq.host_tensor(out)
    qt = llmq.qtensor_view(q, s)
    lib.q_llama_clear_error()
    lib.qmatmul(C.byref(ta), C.byref(qt), C.byref(tc))
    assert lib.q_llama_last_error() == 1  # LLMQ_ERR_ARG
    lib.q_llama_clear_error()


@pytest.mark.skipif(has_gpu(), reason="checks the no-GPU failure path")
def test_no_gpu_fails_loudly(lib):
    """Without a GPU the library reports an error; it never computes on the CPU."""
    A = np.ones((1, 4), np.float32)
    out = np.full((1, 3), 7.0, np.float32)
    q = np.ones((4, 3), np.int8)
    s = np.ones(3, np.float32)
    ta, tc = llmq.host_tensor(A), llmq.host_tensor(out)
    qt = llmq.qtensor_view(q, s)
    lib.q_llama_clear_error()
    lib.qmatmul(C.byref(ta), C.byref(qt), C.byref(tc))
    assert lib.q_llama_last_error() == 3  # LLMQ_ERR_NO_DEVICE
    assert np.all(out == 7.0)
    lib.q_llama_clear_error()
    m = llmq.QLlamaModel()
    assert lib.q_llama_model_load(os.path.join(GOLDEN, "mini.llmq").encode(), C.byref(m)) == 1
    lib.q_llama_clear_error()
    # the attention-path query needs the device's shared-memory limit
    assert lib.llmq_attention_launches(32, 8, 128, 768) == -1
    lib.q_llama_clear_error()


def test_save_roundtrip_and_reference_loader(lib, orc, ref, tmp_path):
    cfg = dict(vocab=96, d_model=32, n_layers=2, n_heads=4, n_kv=2, head_dim=8, d_ff=48, max_seq=40,
               rope_base=10000.0, eps=1e-5)
    m = synth(lib, cfg, seed=9, with_bias=True)
    p = str(tmp_path / "s.llmq")
    assert lib.q_llama_model_save(p.encode(), C.byref(m)) == 0
    assert not os.path.exists(p + ".tmp")
    for loader, free in ((orc.orc_model_load, orc.orc_model_free), (ref.q_llama_model_load, ref.q_llama_model_free)):
        m2 = llmq.QLlamaModel()
        assert loader(p.encode(), C.byref(m2)) == 0
        assert_models_equal(m, m2)
        free(C.byref(m2))
    lib.q_llama_model_free(C.byref(m))


def test_synth_is_seeded_and_follows_the_quantisation_rule(lib):
    cfg = dict(vocab=64, d_model=48, n_layers=1, n_heads=2, n_kv=1, head_dim=24, d_ff=72, max_seq=16,
               rope_base=10000.0, eps=1e-5)
    a, b, c = synth(lib, cfg, seed=1), synth(lib, cfg, seed=1), synth(lib, cfg, seed=2)
    assert_models_equal(a, b)
    qa, _ = llmq.qtensor_arrays(a.blocks[0].Wq)
    qc, _ = llmq.qtensor_arrays(c.blocks[0].Wq)
    assert not np.array_equal(qa, qc)
    # per-column absmax maps to +-127 exactly (quant.c:17-23)
    for name in ("Wq", "Wk", "Wv", "Wo", "Wgate", "Wup", "Wdown"):
        q, s = llmq.qtensor_arrays(getattr(a.blocks[0], name))
        assert np.all(np.abs(q).max(axis=0) == 127), name
        assert np.all(s > 0)
    # weights look like N(0, 0.02): dequantised std within a few percent
    q, s = llmq.qtensor_arrays(a.lm_head)
    w = q.astype(np.float64) * s[None, :]
    assert abs(w.std() - 0.02) < 0.002
    np.testing.assert_array_equal(llmq.vec_array(a.blocks[0].b_q), 0.0)
    np.testing.assert_array_equal(llmq.vec_array(a.blocks[0].attn_norm), 1.0)
    for m in (a, b, c):
        lib.q_llama_model_free(C.byref(m))


def test_link_check_compiles_against_the_reference_headers(tmp_path):
    """A C caller that includes the reference's own tensor.h, quant.h, llama.h
    and sampler.h, then llmq_cuda.h, compiles with -Werror (every shared
    declaration agrees, the include guards interlock) and links against
    libllmq_cuda.so alone (every call resolves in this library)."""
    from conftest import reference_dir
    ref = reference_dir()
    if ref is None:
        pytest.skip("no reference checkout on this machine")
    r = subprocess.run(["make", "-C", os.path.join(ROOT, "tests"), f"REF={ref}", f"OUT={tmp_path}"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert os.access(tmp_path / "link_check", os.X_OK)


@pytest.mark.parametrize("with_bias,fast", [(False, False), (True, False), (False, True)])
def test_streaming_synth_writer_matches_whole_model_save(lib, tmp_path, with_bias, fast):
    """llmq_synth_model_save writes the synthetic model tensor by tensor; the
    file is byte for byte what q_llama_model_save writes for the whole model
    built in memory (tools/convert_llama.py:73-97 layout)."""
    cfg = dict(vocab=300, d_model=64, n_layers=2, n_heads=4, n_kv=2, head_dim=16, d_ff=96, max_seq=32,
               rope_base=10000.0, eps=1e-5)
    c = llmq.config(**cfg)
    m = llmq.QLlamaModel()
    if fast:
        assert lib.llmq_synth_model_fast_shard(C.byref(c), 77, 0, 1, C.byref(m)) == 0
    else:
        assert lib.llmq_synth_model(C.byref(c), 77, 0.02, int(with_bias), C.byref(m)) == 0
    whole, streamed = tmp_path / "whole.llmq", tmp_path / "streamed.llmq"
    assert lib.q_llama_model_save(str(whole).encode(), C.byref(m)) == 0
    assert lib.llmq_synth_model_save(C.byref(c), 77, 0.02, int(with_bias), int(fast), str(streamed).encode()) == 0
    assert whole.read_bytes() == streamed.read_bytes()
    assert not (tmp_path / "streamed.llmq.tmp").exists()
    lib.q_llama_model_free(C.byref(m))


def _llma_v2_bytes(cfg, rng, bias=True):
    """An LLMA v2 file (llama.c:192-269 layout) with random tensors and zero
    biases, and the v1 file it came from (the same without the biases)."""
    V, dm, L, H, KV, hd, dff, ms = (cfg[k] for k in ("vocab", "d_model", "n_layers", "n_heads", "n_kv", "head_dim",
                                                      "d_ff", "max_seq"))
    qd, kvd = H * hd, KV * hd
    f32 = lambda n: rng.standard_normal(n).astype("<f4").tobytes()  # noqa: E731
    head = struct.pack("<8i", V, dm, L, H, KV, hd, dff, ms) + struct.pack("<2f", 10000.0, 1e-5)
    v1, v2 = [struct.pack("<II", 0x414D4C4C, 1) + head], [struct.pack("<II", 0x414D4C4C, 2) + head]
    wte = f32(V * dm)
    v1.append(wte)
    v2.append(wte)
    for _ in range(L):
        pre = f32(dm) + f32(dm * qd) + f32(dm * kvd) + f32(dm * kvd)
        post = f32(qd * dm) + f32(dm) + f32(dm * dff) + f32(dm * dff) + f32(dff * dm)
        v1 += [pre, post]
        v2 += [pre, b"\0" * 4 * (qd + 2 * kvd), post]
    tail = f32(dm) + f32(dm * V)
    v1.append(tail)
    v2.append(tail)
    return b"".join(v1), b"".join(v2)


def test_llma_upgrade_v1_to_v2(lib, tmp_path):
    """llmq_llma_upgrade_v1 (and `llmq_run upgrade-llma`) turns an LLMA v1 file
    into v2 with zero q/k/v biases (tools/upgrade_llma.py), and refuses the
    files the tool refuses."""
    cfg = dict(vocab=50, d_model=16, n_layers=3, n_heads=4, n_kv=2, head_dim=4, d_ff=24, max_seq=16)
    v1, v2 = _llma_v2_bytes(cfg, np.random.default_rng(4))
    src, dst = tmp_path / "v1.bin", tmp_path / "v2.bin"
    src.write_bytes(v1)
    assert lib.llmq_llma_upgrade_v1(str(src).encode(), str(dst).encode()) == 0
    assert dst.read_bytes() == v2
    cli = os.path.join(ROOT, "llm-project_b200", "bin", "llmq_run")
    r = subprocess.run([cli, "upgrade-llma", str(src), str(tmp_path / "cli.bin")], capture_output=True, text=True)
    assert r.returncode == 0 and (tmp_path / "cli.bin").read_bytes() == v2
    for bad, msg in ((v2, b"already version 2"), (b"XXXX" + v1[4:], b"not an LLMA"), (v1[:-4], b"truncated"),
                     (v1 + b"\0", b"trailing bytes"), (v1[:20], b"too small")):
        src.write_bytes(bad)
        r = subprocess.run([cli, "upgrade-llma", str(src), str(tmp_path / "bad.bin")], capture_output=True)
        assert r.returncode == 1 and msg in r.stderr, (msg, r.stderr)
        assert not (tmp_path / "bad.bin").exists()


def test_llma_upgrade_matches_the_reference_tool(lib, tmp_path):
    """Byte for byte what the reference's own tools/upgrade_llma.py writes (run
    where a reference checkout is present)."""
    from conftest import reference_dir
    ref = reference_dir()
    if ref is None or not os.path.exists(os.path.join(ref, "tools", "upgrade_llma.py")):
        pytest.skip("no reference checkout on this machine")
    cfg = dict(vocab=40, d_model=8, n_layers=2, n_heads=2, n_kv=1, head_dim=4, d_ff=12, max_seq=8)
    v1, _ = _llma_v2_bytes(cfg, np.random.default_rng(9))
    src = tmp_path / "v1.bin"
    src.write_bytes(v1)
    r = subprocess.run([sys.executable, os.path.join(ref, "tools", "upgrade_llma.py"), str(src),
                        str(tmp_path / "ref.bin")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert lib.llmq_llma_upgrade_v1(str(src).encode(), str(tmp_path / "ours.bin").encode()) == 0
    assert (tmp_path / "ours.bin").read_bytes() == (tmp_path / "ref.bin").read_bytes()
