"""TEST INFRASTRUCTURE ONLY: Python access to the CPU checkers.

* `load_oracle()`: our C restatement of the reference path (llmq_oracle.c).
* `load_synth()`: the seeded synthetic-model generator built on its own
  (oracle/_build/libsynth.so), the reference arm's input maker.
* `load_reference()`: the reference's own quant.c / matrix.c / llama.c /
  rmsnorm.c / rope.c / gqa.c / swiglu.c / tensor.c / sampler.c, compiled here
  by oracle/Makefile into oracle/_ref/ (None when not built).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module.  The struct layouts come from the product's ctypes binding (llmq.py),
which mirrors the reference headers.
"""
from __future__ import annotations

import ctypes as C
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "llm-project_b200"))

import llmq  # noqa: E402
from llmq import (LlamaKV, LlamaModel, QLlamaModel, QTensor, Rng, Tensor, c_byte_p,  # noqa: E402
                  c_float_p, c_int_p)

ORACLE_PATH = os.path.join(HERE, "_build", "liboracle.so")
SYNTH_PATH = os.path.join(HERE, "_build", "libsynth.so")
REF_DIR = os.path.join(HERE, "_ref")


def _cpu_flags() -> set[str]:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def reference_path() -> str | None:
    """The reference build for this CPU: AVX-512 (x86-64-v4) when available."""
    flags = _cpu_flags()
    v4 = os.path.join(REF_DIR, "libllmq_ref_v4.so")
    v3 = os.path.join(REF_DIR, "libllmq_ref_v3.so")
    if {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"} <= flags and os.path.exists(v4):
        return v4
    if {"avx2", "fma", "bmi2"} <= flags and os.path.exists(v3):
        return v3
    return None


_ORC_SIGS = {
    "orc_quantize_int8_percol": (None, [c_float_p, C.c_int, C.c_int, c_byte_p, c_float_p]),
    "orc_dequantize_int8_percol": (None, [c_byte_p, c_float_p, C.c_int, C.c_int, c_float_p]),
    "orc_quantize_row": (C.c_float, [c_float_p, C.c_int, c_byte_p]),
    "orc_qacc_columns": (None, [c_byte_p, c_byte_p, C.c_int, C.c_int, c_int_p]),
    "orc_qmatmul": (None, [c_float_p, C.c_int, C.c_int, c_byte_p, c_float_p, C.c_int, c_float_p]),
    "orc_rmsnorm_row": (None, [c_float_p, c_float_p, C.c_int, C.c_float, c_float_p]),
    "orc_rope_heads_pos_row": (None, [c_float_p, C.c_int, C.c_int, C.c_float, C.c_int]),
    "orc_argmax": (C.c_int, [c_float_p, C.c_int]),
    "orc_xorshift64": (C.c_ulonglong, [C.POINTER(C.c_ulonglong)]),
    "orc_sample_token": (C.c_int, [c_float_p, C.c_int, C.c_float, C.c_int, C.c_float, C.POINTER(C.c_ulonglong)]),
    "orc_kv_create": (LlamaKV, [C.POINTER(QLlamaModel)]),
    "orc_kv_free": (None, [C.POINTER(LlamaKV)]),
    "orc_decode_step": (None, [C.POINTER(QLlamaModel), C.POINTER(LlamaKV), C.c_int, c_float_p]),
    "orc_f32_kv_create": (LlamaKV, [C.POINTER(LlamaModel)]),
    "orc_f32_decode_step": (None, [C.POINTER(LlamaModel), C.POINTER(LlamaKV), C.c_int, c_float_p]),
    "orc_model_load": (C.c_int, [C.c_char_p, C.POINTER(QLlamaModel)]),
    "orc_model_free": (None, [C.POINTER(QLlamaModel)]),
    "orc_model_save": (C.c_int, [C.c_char_p, C.POINTER(QLlamaModel)]),
    "orc_expf_bits": (None, [C.c_uint32, C.c_uint64, c_float_p]),
    "orc_quantize_from": (QLlamaModel, [C.POINTER(LlamaModel)]),
}

_REF_SIGS = {
    "quantize_int8_percol": (None, [c_float_p, C.c_int, C.c_int, c_byte_p, c_float_p]),
    "dequantize_int8_percol": (None, [c_byte_p, c_float_p, C.c_int, C.c_int, c_float_p]),
    "qmatmul": (None, [C.POINTER(Tensor), C.POINTER(QTensor), C.POINTER(Tensor)]),
    "qacc_columns": (None, [c_byte_p, c_byte_p, C.c_int, C.c_int, c_int_p]),
    "q_llama_model_load": (C.c_int, [C.c_char_p, C.POINTER(QLlamaModel)]),
    "q_llama_model_free": (None, [C.POINTER(QLlamaModel)]),
    "q_llama_quantize_from": (QLlamaModel, [C.POINTER(LlamaModel)]),
    "q_llama_kv_create": (LlamaKV, [C.POINTER(QLlamaModel)]),
    "llama_kv_free": (None, [C.POINTER(LlamaKV)]),
    "q_llama_decode_step": (None, [C.POINTER(QLlamaModel), C.POINTER(LlamaKV), C.c_int, C.POINTER(Tensor)]),
    "llama_model_create": (LlamaModel, [C.c_int] * 8 + [C.c_float, C.c_float]),
    "llama_model_randomize": (None, [C.POINTER(LlamaModel)]),
    "llama_model_forward": (None, [C.POINTER(LlamaModel), c_int_p, C.c_int, C.POINTER(Tensor)]),
    "llama_model_free": (None, [C.POINTER(LlamaModel)]),
    "llama_kv_create": (LlamaKV, [C.POINTER(LlamaModel)]),
    "llama_decode_step": (None, [C.POINTER(LlamaModel), C.POINTER(LlamaKV), C.c_int, C.POINTER(Tensor)]),
    "llama_model_load": (C.c_int, [C.c_char_p, C.POINTER(LlamaModel)]),
    "sample_argmax": (C.c_int, [C.POINTER(Tensor), C.c_int]),
    "rng_create": (Rng, [C.c_ulonglong]),
    "rng_uniform": (C.c_float, [C.POINTER(Rng)]),
    "sample_token": (C.c_int, [C.POINTER(Tensor), C.c_int, C.c_float, C.c_int, C.c_float, C.POINTER(Rng)]),
    "rmsnorm": (None, [C.POINTER(Tensor), C.POINTER(Tensor), C.POINTER(Tensor), C.c_float]),
    "rope_heads_pos": (None, [C.POINTER(Tensor), C.c_int, C.c_float, C.c_int]),
}


def _bind(lib, sigs):
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_cache: dict[str, C.CDLL] = {}


def load_oracle() -> C.CDLL:
    if "orc" not in _cache:
        if not os.path.exists(ORACLE_PATH):
            raise FileNotFoundError(f"{ORACLE_PATH} not built (make -C oracle)")
        _cache["orc"] = _bind(C.CDLL(ORACLE_PATH), _ORC_SIGS)
    return _cache["orc"]


_SYNTH_SIGS = {
    "llmq_synth_model": (C.c_int, [C.POINTER(llmq.LlmqConfig), C.c_uint64, C.c_float, C.c_int,
                                   C.POINTER(QLlamaModel)]),
    "llmq_synth_model_fast_shard": (C.c_int, [C.POINTER(llmq.LlmqConfig), C.c_uint64, C.c_int, C.c_int,
                                              C.POINTER(QLlamaModel)]),
    "llmq_synth_qtensor": (None, [C.POINTER(QTensor), C.c_uint64]),
    "qtensor_create": (QTensor, [C.c_int, C.c_int]),
}


def load_synth() -> C.CDLL:
    """The synthetic-model generator without the product library: the same
    source (llmq_synth.c) built into oracle/_build/libsynth.so.  Its models are
    malloc'd like the reference's, so ref.q_llama_model_free releases them."""
    if "synth" not in _cache:
        if not os.path.exists(SYNTH_PATH):
            raise FileNotFoundError(f"{SYNTH_PATH} not built (make -C oracle)")
        _cache["synth"] = _bind(C.CDLL(SYNTH_PATH), _SYNTH_SIGS)
    return _cache["synth"]


def load_reference() -> C.CDLL | None:
    if "ref" not in _cache:
        p = reference_path()
        if p is None:
            return None
        _cache["ref"] = _bind(C.CDLL(p), _REF_SIGS)
    return _cache["ref"]


def libc() -> C.CDLL:
    if "libc" not in _cache:
        _cache["libc"] = C.CDLL("libc.so.6")
    return _cache["libc"]
