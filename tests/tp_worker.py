"""One rank of the tensor-parallel parity check run by test_gpu_tp.py
(launched with torch.distributed.run, one process per GPU, 2, 4 or 8 ranks).

Every rank decodes its shard of the same synthetic model; rank 0 compares the
whole logits rows (gathered by the library on every rank), the greedy ids of
q_llama_generate and the sampled ids of q_llama_generate_sample with the
oracle's single-sequence decode of the whole model, bit for bit, and writes the
verdicts to <out_dir>/tp.json.  The cases are those whose heads, KV heads, d_ff
and vocabulary divide by the group size (8 KV heads: one per rank at 8)."""
from __future__ import annotations

import ctypes as C
import datetime
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path[:0] = [HERE, os.path.join(ROOT, "llm-project_b200"), os.path.join(ROOT, "oracle")]

import numpy as np  # noqa: E402
import torch.distributed as dist  # noqa: E402

import llmq  # noqa: E402
import oracle  # noqa: E402
from helpers import TINY, bits_equal, fp, orc_decode, orc_sample, synth  # noqa: E402

# GQA 16/8, hd 32, with biases: shards at 2, 4 and 8 ranks
GQA8 = dict(vocab=32000, d_model=512, n_layers=3, n_heads=16, n_kv=8, head_dim=32, d_ff=1024, max_seq=128,
            rope_base=10000.0, eps=1e-5)

CASES = [
    ("tiny_bias", TINY, True, [5, 77, 31999, 0, 1234, 42, 9, 17, 256, 3000]),
    ("gqa8_bias", GQA8, True, [5, 77, 31999, 0, 1234, 42, 9, 17]),
    ("8b_shapes_2_layers", dict(vocab=128256, d_model=4096, n_layers=2, n_heads=32, n_kv=8, head_dim=128,
                                d_ff=14336, max_seq=64, rope_base=500000.0, eps=1e-5), False, [17, 128000, 42]),
]


def shardable(cfg, world):
    return all(cfg[k] % world == 0 for k in ("n_heads", "n_kv", "d_ff", "vocab"))


def main():
    out_dir = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    lib = llmq.load()
    if lib.q_llama_set_device(int(os.environ["LOCAL_RANK"])) != 0:
        llmq.check(lib)
    llmq.tp_bootstrap(lib, rank, world)
    verdicts = {}
    for name, cfg, bias, ids in CASES:
        if not shardable(cfg, world):
            continue
        sh = llmq.synth_shard(lib, cfg, 1234, rank, world, with_bias=bias)
        kv = lib.q_llama_kv_create(C.byref(sh))
        llmq.check(lib)
        got = np.zeros((len(ids), cfg["vocab"]), np.float32)
        row = np.zeros((1, cfg["vocab"]), np.float32)
        t = llmq.host_tensor(row)
        for i, tok in enumerate(ids):
            lib.q_llama_decode_step(C.byref(sh), C.byref(kv), int(tok), C.byref(t))
            llmq.check(lib)
            got[i] = row[0]
        n_gen = 6
        gen = (C.c_int * n_gen)()
        if lib.q_llama_generate(C.byref(sh), C.byref(kv), int(np.argmax(got[-1])), n_gen, gen) != 0:
            llmq.check(lib)
        # then sampled steps (temperature 0.8, top-k 40, top-p 0.95, seed 1234),
        # every rank drawing from the gathered row with the same stream
        n_smp = 8
        smp = (C.c_int * n_smp)()
        r = lib.rng_create(1234)
        if lib.q_llama_generate_sample(C.byref(sh), C.byref(kv), gen[n_gen - 1], n_smp, 0.8, 40, 0.95, C.byref(r),
                                       smp) != 0:
            llmq.check(lib)
        if rank == 0:
            orc = oracle.load_oracle()
            full = synth(lib, cfg, seed=1234, with_bias=bias)
            greedy = [int(np.argmax(got[-1]))]
            for _ in range(n_gen):
                greedy.append(int(np.argmax(orc_decode(orc, full, ids + greedy)[0][-1])))
            want, _ = orc_decode(orc, full, ids)
            verdicts[name + ".logits"] = bits_equal(got, want)
            verdicts[name + ".generate"] = list(gen) == greedy[1:]
            kvo = orc.orc_kv_create(C.byref(full))
            row_o = np.zeros(cfg["vocab"], np.float32)
            for tok in ids + greedy[:-1]:
                orc.orc_decode_step(C.byref(full), C.byref(kvo), int(tok), fp(row_o))
            st, tok, want_s = lib.rng_create(1234).state, greedy[-1], []
            for _ in range(n_smp):
                orc.orc_decode_step(C.byref(full), C.byref(kvo), int(tok), fp(row_o))
                tok, st = orc_sample(orc, row_o, 0.8, 40, 0.95, st)
                want_s.append(tok)
            orc.orc_kv_free(C.byref(kvo))
            verdicts[name + ".generate_sample"] = list(smp) == want_s and r.state == st
            lib.q_llama_model_free(C.byref(full))
        dist.barrier()
        lib.llama_kv_free(C.byref(kv))
        lib.q_llama_model_free(C.byref(sh))
    # batched passes on the shards: three prompts of different lengths
    # prefilled, then three batched steps with logits; every row equals the
    # oracle's single-sequence decode of the whole model
    cfg = TINY if shardable(TINY, world) else GQA8
    bname = "tiny_bias" if cfg is TINY else "gqa8_bias"
    sh = llmq.synth_shard(lib, cfg, 1234, rank, world, with_bias=True)
    rng = np.random.default_rng(9)
    lens, steps = [5, 1, 12], 3
    seqs = [rng.integers(0, cfg["vocab"], n + steps).tolist() for n in lens]
    kvs = [lib.q_llama_kv_create(C.byref(sh)) for _ in lens]
    llmq.check(lib)
    firsts = []
    for kv, sq, n in zip(kvs, seqs, lens):
        firsts.append(lib.q_llama_prefill_argmax(C.byref(sh), C.byref(kv), llmq.int_array(sq[:n]), n, None))
        llmq.check(lib)
    got = np.zeros((len(lens), steps, cfg["vocab"]), np.float32)
    for i in range(steps):
        out = np.zeros((len(lens), cfg["vocab"]), np.float32)
        t = llmq.host_tensor(out)
        lib.q_llama_decode_batch(C.byref(sh), llmq.kv_pointers(kvs), llmq.int_array([sq[n + i] for sq, n in zip(seqs, lens)]),
                                 len(lens), C.byref(t))
        llmq.check(lib)
        got[:, i] = out
    if rank == 0:
        orc = oracle.load_oracle()
        full = synth(lib, cfg, seed=1234, with_bias=True)
        ok_rows, ok_first = True, True
        for b, (sq, n) in enumerate(zip(seqs, lens)):
            want, _ = orc_decode(orc, full, sq)
            ok_rows &= bits_equal(got[b], want[n:])
            ok_first &= firsts[b] == int(np.argmax(want[n - 1]))
        verdicts[bname + ".batch_logits"] = bool(ok_rows)
        verdicts[bname + ".prefill_ids"] = bool(ok_first)
        lib.q_llama_model_free(C.byref(full))
    dist.barrier()
    for kv in kvs:
        lib.llama_kv_free(C.byref(kv))
    lib.q_llama_model_free(C.byref(sh))
    dist.barrier()
    lib.q_llama_tp_shutdown()
    if rank == 0:
        with open(os.path.join(out_dir, "tp.json"), "w") as f:
            json.dump(verdicts, f)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
