"""ctypes binding of libllmq_cuda.so for Python callers (tests, bench).

The C entry points keep the names and argument meaning of the reference's
quant.h / llama.h (marjoncajocon/llm-project quant.h:15-33, llama.h:114-140),
so this module mirrors them one to one, plus thin numpy helpers.  There is no
fallback: if the shared library is missing, `load()` raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libllmq_cuda.so")

c_float_p = C.POINTER(C.c_float)
c_int_p = C.POINTER(C.c_int)
c_byte_p = C.POINTER(C.c_byte)


class Tensor(C.Structure):  # tensor.h:10-16
    _fields_ = [("data", c_float_p), ("grad", c_float_p), ("shape", c_int_p), ("ndim", C.c_int),
                ("size", C.c_size_t)]


class Rng(C.Structure):  # sampler.h:13-15
    _fields_ = [("state", C.c_ulonglong)]


class QTensor(C.Structure):  # quant.h:22-26
    _fields_ = [("rows", C.c_int), ("cols", C.c_int), ("q", c_byte_p), ("scale", c_float_p)]


class LlamaBlock(C.Structure):  # llama.h:19-36
    _fields_ = [("d_model", C.c_int), ("n_heads", C.c_int), ("n_kv", C.c_int), ("head_dim", C.c_int),
                ("d_ff", C.c_int), ("rope_base", C.c_float), ("eps", C.c_float)] + \
               [(n, Tensor) for n in ("attn_norm", "Wq", "Wk", "Wv", "b_q", "b_k", "b_v", "Wo",
                                      "ffn_norm", "Wgate", "Wup", "Wdown")]


CONFIG_FIELDS = ("vocab", "d_model", "n_layers", "n_heads", "n_kv", "head_dim", "d_ff", "max_seq")


class LlamaModel(C.Structure):  # llama.h:59-66
    _fields_ = [(n, C.c_int) for n in CONFIG_FIELDS] + \
               [("rope_base", C.c_float), ("eps", C.c_float), ("wte", Tensor),
                ("blocks", C.POINTER(LlamaBlock)), ("final_norm", Tensor), ("lm_head", Tensor)]


class LlamaKV(C.Structure):  # llama.h:94-99
    _fields_ = [("n_layers", C.c_int), ("max_seq", C.c_int), ("kv_dim", C.c_int), ("len", C.c_int),
                ("k", C.POINTER(c_float_p)), ("v", C.POINTER(c_float_p))]


class QLlamaBlock(C.Structure):  # llama.h:114-118
    _fields_ = [(n, Tensor) for n in ("attn_norm", "ffn_norm", "b_q", "b_k", "b_v")] + \
               [(n, QTensor) for n in ("Wq", "Wk", "Wv", "Wo", "Wgate", "Wup", "Wdown")]


class QLlamaModel(C.Structure):  # llama.h:120-127
    _fields_ = [(n, C.c_int) for n in CONFIG_FIELDS] + \
               [("rope_base", C.c_float), ("eps", C.c_float), ("wte", QTensor),
                ("blocks", C.POINTER(QLlamaBlock)), ("final_norm", Tensor), ("lm_head", QTensor)]


class LlmqConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in CONFIG_FIELDS] + [("rope_base", C.c_float), ("eps", C.c_float)]


def config(vocab, d_model, n_layers, n_heads, n_kv, head_dim, d_ff, max_seq, rope_base=10000.0,
           eps=1e-5) -> LlmqConfig:
    return LlmqConfig(vocab, d_model, n_layers, n_heads, n_kv, head_dim, d_ff, max_seq, rope_base, eps)


# Signatures of every exported entry point: name -> (restype, argtypes).
SIGNATURES = {
    "quantize_int8_percol": (None, [c_float_p, C.c_int, C.c_int, c_byte_p, c_float_p]),
    "dequantize_int8_percol": (None, [c_byte_p, c_float_p, C.c_int, C.c_int, c_float_p]),
    "qtensor_create": (QTensor, [C.c_int, C.c_int]),
    "qtensor_free": (None, [C.POINTER(QTensor)]),
    "qtensor_quantize": (None, [C.POINTER(QTensor), c_float_p]),
    "qmatmul": (None, [C.POINTER(Tensor), C.POINTER(QTensor), C.POINTER(Tensor)]),
    "q_llama_model_load": (C.c_int, [C.c_char_p, C.POINTER(QLlamaModel)]),
    "q_llama_model_free": (None, [C.POINTER(QLlamaModel)]),
    "q_llama_quantize_from": (QLlamaModel, [C.POINTER(LlamaModel)]),
    "q_llama_kv_create": (LlamaKV, [C.POINTER(QLlamaModel)]),
    "llama_kv_free": (None, [C.POINTER(LlamaKV)]),
    "q_llama_decode_step": (None, [C.POINTER(QLlamaModel), C.POINTER(LlamaKV), C.c_int, C.POINTER(Tensor)]),
    "q_llama_last_error": (C.c_int, []),
    "q_llama_last_error_message": (C.c_char_p, []),
    "q_llama_clear_error": (None, []),
    "q_llama_decode_step_argmax": (C.c_int, [C.POINTER(QLlamaModel), C.POINTER(LlamaKV), C.c_int,
                                             C.POINTER(Tensor)]),
    "q_llama_kv_sync_host": (C.c_int, [C.POINTER(QLlamaModel), C.POINTER(LlamaKV)]),
    "q_llama_model_save": (C.c_int, [C.c_char_p, C.POINTER(QLlamaModel)]),
    "llmq_synth_model": (C.c_int, [C.POINTER(LlmqConfig), C.c_uint64, C.c_float, C.c_int,
                                   C.POINTER(QLlamaModel)]),
    "llmq_synth_qtensor": (None, [C.POINTER(QTensor), C.c_uint64]),
    "llmq_synth_model_save": (C.c_int, [C.POINTER(LlmqConfig), C.c_uint64, C.c_float, C.c_int, C.c_int, C.c_char_p]),
    "llmq_llma_upgrade_v1": (C.c_int, [C.c_char_p, C.c_char_p]),
    "llmq_synth_model_shard": (C.c_int, [C.POINTER(LlmqConfig), C.c_uint64, C.c_float, C.c_int, C.c_int, C.c_int,
                                         C.POINTER(QLlamaModel)]),
    "llmq_synth_model_fast_shard": (C.c_int, [C.POINTER(LlmqConfig), C.c_uint64, C.c_int, C.c_int,
                                              C.POINTER(QLlamaModel)]),
    "q_llama_model_shard": (C.c_int, [C.POINTER(QLlamaModel), C.c_int, C.c_int, C.POINTER(QLlamaModel)]),
    "q_llama_model_upload": (C.c_int, [C.POINTER(QLlamaModel)]),
    "q_llama_generate": (C.c_int, [C.POINTER(QLlamaModel), C.POINTER(LlamaKV), C.c_int, C.c_int, c_int_p]),
    "llama_kv_create": (LlamaKV, [C.POINTER(LlamaModel)]),
    "llama_decode_step": (None, [C.POINTER(LlamaModel), C.POINTER(LlamaKV), C.c_int, C.POINTER(Tensor)]),
    "llama_decode_step_argmax": (C.c_int, [C.POINTER(LlamaModel), C.POINTER(LlamaKV), C.c_int, C.POINTER(Tensor)]),
    "llama_decode_step_sample": (C.c_int, [C.POINTER(LlamaModel), C.POINTER(LlamaKV), C.c_int, C.c_float, C.c_int,
                                           C.c_float, C.POINTER(Rng), C.POINTER(Tensor)]),
    "llama_generate": (C.c_int, [C.POINTER(LlamaModel), C.POINTER(LlamaKV), C.c_int, C.c_int, c_int_p]),
    "llama_generate_sample": (C.c_int, [C.POINTER(LlamaModel), C.POINTER(LlamaKV), C.c_int, C.c_int, C.c_float,
                                        C.c_int, C.c_float, C.POINTER(Rng), c_int_p]),
    "llmq_llama_model_load": (C.c_int, [C.c_char_p, C.POINTER(LlamaModel)]),
    "llmq_llama_model_free": (None, [C.POINTER(LlamaModel)]),
    "llmq_llama_model_upload": (C.c_int, [C.POINTER(LlamaModel)]),
    "llmq_llama_model_release": (None, [C.POINTER(LlamaModel)]),
    "llmq_synth_model_f32": (C.c_int, [C.POINTER(LlmqConfig), C.c_uint64, C.c_float, C.c_int, C.POINTER(LlamaModel)]),
    "rng_create": (Rng, [C.c_ulonglong]),
    "rng_uniform": (C.c_float, [C.POINTER(Rng)]),
    "sample_argmax": (C.c_int, [C.POINTER(Tensor), C.c_int]),
    "sample_token": (C.c_int, [C.POINTER(Tensor), C.c_int, C.c_float, C.c_int, C.c_float, C.POINTER(Rng)]),
    "q_llama_decode_step_sample": (C.c_int, [C.POINTER(QLlamaModel), C.POINTER(LlamaKV), C.c_int, C.c_float,
                                             C.c_int, C.c_float, C.POINTER(Rng), C.POINTER(Tensor)]),
    "q_llama_generate_sample": (C.c_int, [C.POINTER(QLlamaModel), C.POINTER(LlamaKV), C.c_int, C.c_int,
                                          C.c_float, C.c_int, C.c_float, C.POINTER(Rng), c_int_p]),
    "q_llama_last_step_ms": (C.c_float, []),
    "llmq_expf_device": (C.c_int, [c_float_p, c_float_p, C.c_longlong]),
    "llmq_bench_gemv": (C.c_int, [C.POINTER(QLlamaModel), C.c_int, C.c_int, C.c_int, c_float_p,
                                  C.POINTER(C.c_double)]),
    "llmq_kernels_per_step": (C.c_int, [C.POINTER(QLlamaModel)]),
    "llmq_attention_launches": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "q_llama_set_device": (C.c_int, [C.c_int]),
    "llmq_step_profile": (C.c_int, [C.POINTER(QLlamaModel), C.POINTER(LlamaKV), C.c_int, c_float_p, C.c_int]),
    "qmatmul_device_noalloc": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                         C.c_void_p, C.c_void_p]),
    "llmq_bench_qmatmul": (C.c_int, [C.POINTER(QTensor), C.c_int, C.c_int, c_float_p]),
    "llmq_tp_wait_timeout_check": (C.c_int, [C.c_int, C.c_uint, c_int_p, c_float_p]),
    "llmq_rmsnorm_qmatmul": (C.c_int, [c_float_p, c_float_p, C.c_float, C.POINTER(QTensor), c_float_p]),
    "llmq_spec_sum_check": (C.c_int, [c_float_p, C.c_int, C.c_int, C.c_int, c_float_p, c_int_p,
                                      C.POINTER(C.c_longlong)]),
    "q_llama_decode_batch": (None, [C.POINTER(QLlamaModel), C.POINTER(C.POINTER(LlamaKV)), c_int_p, C.c_int,
                                    C.POINTER(Tensor)]),
    "q_llama_decode_batch_argmax": (C.c_int, [C.POINTER(QLlamaModel), C.POINTER(C.POINTER(LlamaKV)), c_int_p,
                                              C.c_int, c_int_p]),
    "q_llama_prefill": (None, [C.POINTER(QLlamaModel), C.POINTER(LlamaKV), c_int_p, C.c_int, C.POINTER(Tensor)]),
    "llmq_last_launches": (C.c_longlong, []),
    "q_llama_tp_unique_id": (C.c_int, [C.c_char_p]),
    "q_llama_tp_init": (C.c_int, [C.c_int, C.c_int, C.c_char_p]),
    "q_llama_tp_shutdown": (None, []),
    "q_llama_prefill_argmax": (C.c_int, [C.POINTER(QLlamaModel), C.POINTER(LlamaKV), c_int_p, C.c_int,
                                         C.POINTER(Tensor)]),
}

_lib = None


def load(path: str | None = None) -> C.CDLL:
    """Load libllmq_cuda.so and declare its signatures.  Raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise FileNotFoundError(f"{p} not built: run __graft_entry__.build() (make -C llm-project_b200/csrc)")
    lib = C.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


# error codes (llmq_cuda.h)
LLMQ_OK, LLMQ_ERR_ARG, LLMQ_ERR_CUDA, LLMQ_ERR_NO_DEVICE, LLMQ_ERR_IO, LLMQ_ERR_OOM, LLMQ_ERR_STATE = range(7)


class LlmqError(RuntimeError):
    pass


def check(lib) -> None:
    """Raise LlmqError if the last call on this thread failed."""
    code = lib.q_llama_last_error()
    if code != 0:
        msg = lib.q_llama_last_error_message().decode(errors="replace")
        lib.q_llama_clear_error()
        raise LlmqError(f"libllmq_cuda error {code}: {msg}")


# ---------------------------------------------------------------- numpy views
def host_tensor(arr: np.ndarray) -> Tensor:
    """A Tensor struct viewing a C-contiguous float32 numpy array (no copy)."""
    assert arr.dtype == np.float32 and arr.flags["C_CONTIGUOUS"]
    shape = (C.c_int * arr.ndim)(*arr.shape)
    t = Tensor(arr.ctypes.data_as(c_float_p), None, C.cast(shape, c_int_p), arr.ndim, arr.size)
    t._keep = (arr, shape)  # keep the buffers alive with the struct
    return t


def qtensor_view(q: np.ndarray, scale: np.ndarray) -> QTensor:
    """A QTensor struct viewing int8 codes (rows, cols) and f32 scales (cols)."""
    assert q.dtype == np.int8 and q.flags["C_CONTIGUOUS"] and q.ndim == 2
    assert scale.dtype == np.float32 and scale.shape == (q.shape[1],)
    t = QTensor(q.shape[0], q.shape[1], q.ctypes.data_as(c_byte_p), scale.ctypes.data_as(c_float_p))
    t._keep = (q, scale)
    return t


def qtensor_arrays(t: QTensor) -> tuple[np.ndarray, np.ndarray]:
    """numpy copies of a QTensor's codes and scales."""
    q = np.ctypeslib.as_array(C.cast(t.q, c_byte_p), shape=(t.rows * t.cols,)).astype(np.int8)
    s = np.ctypeslib.as_array(t.scale, shape=(t.cols,)).copy()
    return q.reshape(t.rows, t.cols).copy(), s


def kv_pointers(kvs) -> C.Array:
    """A LlamaKV*[] array for the batched entry points (the structs stay owned
    by the caller and must outlive the call)."""
    arr = (C.POINTER(LlamaKV) * len(kvs))(*[C.pointer(k) for k in kvs])
    return arr


def int_array(vals) -> C.Array:
    return (C.c_int * len(vals))(*[int(v) for v in vals])


def tp_bootstrap(lib, rank: int, world: int) -> None:
    """Forms the tensor-parallel group: rank 0 makes the NCCL id, the ranks'
    torch.distributed process group (any backend) broadcasts its 128 bytes,
    every rank joins with q_llama_tp_init.  Call after q_llama_set_device."""
    import torch
    import torch.distributed as dist
    buf = C.create_string_buffer(128)
    if rank == 0 and lib.q_llama_tp_unique_id(buf) != 0:
        check(lib)
    t = torch.tensor(list(buf.raw), dtype=torch.uint8)
    dist.broadcast(t, 0)
    if lib.q_llama_tp_init(rank, world, bytes(t.tolist())) != 0:
        check(lib)


def synth_shard(lib, cfg: dict, seed: int, rank: int, world: int, stddev=0.02, with_bias=False) -> QLlamaModel:
    m = QLlamaModel()
    c = config(**cfg)
    if lib.llmq_synth_model_shard(C.byref(c), seed, stddev, 1 if with_bias else 0, rank, world, C.byref(m)) != 0:
        check(lib)
    return m


def vec_array(t: Tensor) -> np.ndarray:
    return np.ctypeslib.as_array(t.data, shape=(t.size,)).copy()


def model_config(m: QLlamaModel) -> dict:
    d = {n: getattr(m, n) for n in CONFIG_FIELDS}
    d["rope_base"] = m.rope_base
    d["eps"] = m.eps
    return d
