"""Host side of tensor parallelism, on CPU: the shard generator and the
shard cutter give the same tensors, every shard equals the matching slice of
the whole model (row shards keep the whole columns' scales), and a 2-rank gloo
group bootstraps the NCCL id the way the GPU ranks do."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

import llmq
from helpers import assert_models_equal, model_arrays, synth

CFG = dict(vocab=512, d_model=64, n_layers=2, n_heads=4, n_kv=2, head_dim=16, d_ff=160, max_seq=32,
           rope_base=10000.0, eps=1e-5)


@pytest.mark.parametrize("world", [2])
def test_shards_are_slices_of_the_whole_model(lib, world):
    full = synth(lib, CFG, seed=17, with_bias=True)
    F = model_arrays(full)
    hd = CFG["head_dim"]
    qd, kvd, dff, V = CFG["n_heads"] * hd, CFG["n_kv"] * hd, CFG["d_ff"], CFG["vocab"]
    for rank in range(world):
        sh = llmq.synth_shard(lib, CFG, 17, rank, world, with_bias=True)
        cut = llmq.QLlamaModel()
        assert lib.q_llama_model_shard(C.byref(full), rank, world, C.byref(cut)) == 0
        assert_models_equal(sh, cut)
        S = model_arrays(sh)
        cols = {"Wq": qd // world, "Wk": kvd // world, "Wv": kvd // world, "Wgate": dff // world,
                "Wup": dff // world}
        for l in range(CFG["n_layers"]):
            for n, w in cols.items():
                q, s = F[f"{l}.{n}"]
                np.testing.assert_array_equal(S[f"{l}.{n}"][0], q[:, rank * w:(rank + 1) * w])
                np.testing.assert_array_equal(S[f"{l}.{n}"][1], s[rank * w:(rank + 1) * w])
            for n, h in (("Wo", qd // world), ("Wdown", dff // world)):
                q, s = F[f"{l}.{n}"]
                np.testing.assert_array_equal(S[f"{l}.{n}"][0], q[rank * h:(rank + 1) * h])
                np.testing.assert_array_equal(S[f"{l}.{n}"][1], s)  # the whole columns' scales
            for n, w in (("b_q", qd // world), ("b_k", kvd // world), ("b_v", kvd // world)):
                np.testing.assert_array_equal(S[f"{l}.{n}"], F[f"{l}.{n}"][rank * w:(rank + 1) * w])
        q, s = F["lm_head"]
        w = V // world
        np.testing.assert_array_equal(S["lm_head"][0], q[:, rank * w:(rank + 1) * w])
        np.testing.assert_array_equal(S["wte"][0], F["wte"][0])
        lib.q_llama_model_free(C.byref(sh))
        lib.q_llama_model_free(C.byref(cut))
    lib.q_llama_model_free(C.byref(full))


def test_row_shards_add_up_to_the_whole_product(lib, orc):
    """The row-parallel identity the GPU ranks rely on: with the activation scale
    of the whole row, the int32 partial sums of the row shards add up to the
    whole product's sums (checked against the oracle's qmatmul)."""
    rng = np.random.default_rng(3)
    K, N, W = 96, 40, 2
    A = rng.standard_normal((1, K)).astype(np.float32)
    q = rng.integers(-127, 128, size=(K, N)).astype(np.int8)
    s = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    m = np.float32(np.max(np.abs(A)))
    a_s = np.float32(m / np.float32(127.0))
    inv = np.float32(np.float32(1.0) / a_s)
    codes = np.clip(np.rint(A[0] * inv), -127, 127).astype(np.int32)  # ties: no exact .5 in this draw
    parts = [codes[r * K // W:(r + 1) * K // W] @ q[r * K // W:(r + 1) * K // W].astype(np.int32) for r in range(W)]
    acc = np.sum(parts, axis=0).astype(np.int32)
    y = (a_s * s).astype(np.float32) * acc.astype(np.float32)
    out = np.zeros((1, N), np.float32)
    orc.orc_qmatmul(A.ctypes.data_as(llmq.c_float_p), 1, K, q.ctypes.data_as(llmq.c_byte_p),
                    s.ctypes.data_as(llmq.c_float_p), N, out.ctypes.data_as(llmq.c_float_p))
    np.testing.assert_array_equal(y.view(np.uint32), out[0].view(np.uint32))


def _bootstrap_rank(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lib = llmq.load()
    import torch
    buf = C.create_string_buffer(128)
    if rank == 0:
        assert lib.q_llama_tp_unique_id(buf) == 0
    t = torch.tensor(list(buf.raw), dtype=torch.uint8)
    dist.broadcast(t, 0)
    sh = llmq.synth_shard(lib, CFG, 17, rank, world)
    S = model_arrays(sh)
    digest = np.frombuffer(S["0.Wo"][0].tobytes(), np.uint8).astype(np.int64).sum()
    with open(os.path.join(out_dir, f"r{rank}"), "w") as f:
        f.write(bytes(t.tolist()).hex() + " " + str(int(digest)))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks_share_the_nccl_id(tmp_path):
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    mp.start_processes(_bootstrap_rank, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    r0, r1 = (open(tmp_path / f"r{i}").read().split() for i in range(2))
    assert r0[0] == r1[0] and r0[0] != "00" * 128  # one id, not empty
    assert r0[1] != r1[1]  # the two Wo row shards differ
