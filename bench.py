"""Benchmark: int8 (W8A8) LLaMA-family KV-cache decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload 8b|8b2|tiny|serve64|serve16-2l|serve64-tp|70b|70b-bs32|sweep]

Default workload: LLaMA-3-8B-shaped int8 model
(dm 4096, 32 layers, 32/8 heads, hd 128, dff 14336, vocab 128256, rope 5e5),
synthetic seeded N(0, 0.02) weights quantised per column, batch 1, a 512-id
uniform-random prompt, then greedy decode.  A step is one decoded token.

Our arm prints one JSON line with
  value     tok/s of K greedy steps chained on the GPU (inputs resident in HBM,
            one CUDA graph per step, timed with CUDA events on the model stream)
  e2e       tok/s of the same K positions through q_llama_decode_step (the
            reference API): token in from the host, f32 logits back to the host,
            host argmax; wall clock
  roofline  the int8 GEMV kernel (k_gemv, the dominant kernel): algorithmic bytes
            / CUDA-event time per launch, over the step's launch mix
  cpu_baseline  the reference's own q_llama_decode_step (oracle/_ref, all host
            cores) on the same model and KV cache, on a bounded sample of steps
and, on one GPU, the other configs as objects of the same line:
  bs64      configs[3]: 64 sequences x 2048-id prompts prefilled, then a bounded
            number of batched greedy decode steps (tok/s, prefill tok/s, e2e)
  tiny      configs[0]: the tiny model, 16-id prompt + 240 greedy tokens, GPU
            us/token beside the reference's CPU decode of the same tokens
  gemv_sweep  configs[1]: isolated products, M = 1, 8, 64, 256, with the
            reference's CPU qmatmul time beside each
With N > 1 every rank runs an independent replica of the bs1 decode (weak
scaling, max over ranks) and then, under `tp`, the same model and prompt as one
tensor-parallel group of all N GPUs, whose greedy ids must equal the 1-GPU run's.
`--impl reference` times the reference's CPU decode alone on the same config
(its inputs come from oracle/_build/libsynth.so: no library of ours is mapped).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "llm-project_b200"))
import llmq  # noqa: E402

WORKLOADS = {
    "8b": dict(cfg=dict(vocab=128256, d_model=4096, n_layers=32, n_heads=32, n_kv=8, head_dim=128, d_ff=14336,
                        rope_base=500000.0, eps=1e-5), prompt=512, gen=256,
               name="llama3-8b-shaped int8 W8A8, batch 1: 512-id prompt then greedy decode"),
    "8b2": dict(cfg=dict(vocab=128256, d_model=4096, n_layers=2, n_heads=32, n_kv=8, head_dim=128, d_ff=14336,
                         rope_base=500000.0, eps=1e-5), prompt=512, gen=256,
                name="llama3-8b layer shapes, 2 layers (profiling case), batch 1"),
    "serve64": dict(cfg=dict(vocab=128256, d_model=4096, n_layers=32, n_heads=32, n_kv=8, head_dim=128,
                             d_ff=14336, rope_base=500000.0, eps=1e-5), prompt=2048, gen=128, batch=64,
                    name="llama3-8b-shaped int8 W8A8 batched serving: 64 sequences, 2048-id prompts prefilled, "
                         "then batched greedy decode"),
    "serve16-2l": dict(cfg=dict(vocab=128256, d_model=4096, n_layers=2, n_heads=32, n_kv=8, head_dim=128,
                                d_ff=14336, rope_base=500000.0, eps=1e-5), prompt=1024, gen=8, batch=16,
                       name="llama3-8b layer shapes, 2 layers (profiling case): 16 sequences, 1024-id prompts "
                            "prefilled, then batched greedy decode"),
    "70b": dict(cfg=dict(vocab=128256, d_model=8192, n_layers=80, n_heads=64, n_kv=8, head_dim=128, d_ff=28672,
                         rope_base=500000.0, eps=1e-5), prompt=1024, gen=256, tp=True, fast=True,
                name="llama3-70b-shaped int8 W8A8, batch 1, tensor-parallel over all GPUs: 1024-id prompt then "
                     "greedy decode"),
    "serve64-tp": dict(cfg=dict(vocab=128256, d_model=4096, n_layers=32, n_heads=32, n_kv=8, head_dim=128,
                                d_ff=14336, rope_base=500000.0, eps=1e-5), prompt=2048, gen=128, batch=64, tp=True,
                       name="llama3-8b-shaped int8 W8A8 batched serving, tensor-parallel over all GPUs: 64 sequences, "
                            "2048-id prompts prefilled, then batched greedy decode"),
    "70b-bs32": dict(cfg=dict(vocab=128256, d_model=8192, n_layers=80, n_heads=64, n_kv=8, head_dim=128,
                              d_ff=28672, rope_base=500000.0, eps=1e-5), prompt=1024, gen=256, batch=32, tp=True,
                     fast=True,
                     name="llama3-70b-shaped int8 W8A8, batch 32, tensor-parallel over all GPUs: 1024-id prompts "
                          "prefilled, then batched greedy decode"),
    "8b-f32": dict(cfg=dict(vocab=128256, d_model=4096, n_layers=32, n_heads=32, n_kv=8, head_dim=128, d_ff=14336,
                            rope_base=500000.0, eps=1e-5), prompt=64, gen=128, f32=True,
                   name="llama3-8b-shaped fp32 (LLMA path: the int8 synthetic model dequantised, as "
                        "llama_model_load reads an LLMQ file), batch 1: 64-id prompt then greedy decode"),
    "8b2-f32": dict(cfg=dict(vocab=128256, d_model=4096, n_layers=2, n_heads=32, n_kv=8, head_dim=128,
                             d_ff=14336, rope_base=500000.0, eps=1e-5), prompt=16, gen=64, f32=True,
                    name="llama3-8b layer shapes in fp32, 2 layers (profiling case), batch 1"),
    "tiny": dict(cfg=dict(vocab=32000, d_model=288, n_layers=6, n_heads=6, n_kv=2, head_dim=48, d_ff=768,
                          rope_base=10000.0, eps=1e-5), prompt=16, gen=240,
                 name="tiny llama int8 W8A8, batch 1: 16-id prompt then greedy decode"),
}
SEED_WEIGHTS, SEED_PROMPT = 1234, 5678
METRIC = "int8-weight decode tok/s (bs1)"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons with NVML every ~20 ms."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # pragma: no cover - reported in the JSON
            self.error = str(e)

    def _run(self):
        nv = self._nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = get_reasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._h is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# -------------------------------------------------------------- model setup
def make_model(lib, cfg: dict, max_seq: int):
    c = llmq.config(max_seq=max_seq, **cfg)
    m = llmq.QLlamaModel()
    t0 = time.time()
    rc = lib.llmq_synth_model(C.byref(c), SEED_WEIGHTS, 0.02, 0, C.byref(m))
    if rc != 0:
        raise RuntimeError(lib.q_llama_last_error_message().decode())
    log(f"synthetic model built in {time.time() - t0:.1f}s")
    return m


def weight_bytes(cfg: dict) -> int:
    dm, L, qd = cfg["d_model"], cfg["n_layers"], cfg["n_heads"] * cfg["head_dim"]
    kvd, dff, V = cfg["n_kv"] * cfg["head_dim"], cfg["d_ff"], cfg["vocab"]
    per_layer = dm * (qd + 2 * kvd) + qd * dm + 2 * dm * dff + dff * dm
    return L * per_layer + dm * V


def prompt_ids(cfg, n):
    return np.random.default_rng(SEED_PROMPT).integers(0, cfg["vocab"], size=n).astype(np.int32)


# ---------------------------------------------------------------- our arm
def bs1_config(args, wl, P, W, K, world):
    """The `config` of a batch-1 line; both arms print this same dict."""
    step_bytes = weight_bytes(wl["cfg"])
    if step_bytes > 126e6:
        l2 = f"inputs larger than L2: {step_bytes / 1e9:.2f} GB of int8 weights streamed per step"
    else:
        l2 = f"{step_bytes / 1e6:.1f} MB of int8 weights fit in the 126 MB L2: a latency-bound step, no flush"
    return {"workload": wl["name"], "model": f"{args.workload}-shaped synthetic, seed {SEED_WEIGHTS}",
            "global_batch": world, "batch_per_gpu": 1, "prompt": P, "kv_len_start": P + W,
            "kv_len_end": P + W + K,
            "parallelism": "single GPU" if world == 1 else f"{world} independent replicas",
            "l2": l2,
            "prompt_cache": f"our arm decodes the {P} prompt ids on the GPU; the reference arm fills the prompt's "
                            f"cache rows with seeded values instead (decoding a long prompt on the CPU takes "
                            f"minutes); the timed steps of both attend over the same positions"}


def max_over_ranks(vals, dist):
    if dist is None:
        return vals
    import torch
    t = torch.tensor(vals, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def run_ours(args, rank, world):
    lib = llmq.load()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if lib.q_llama_set_device(local) != 0:
        raise RuntimeError(lib.q_llama_last_error_message().decode())
    wl = WORKLOADS[args.workload]
    cfg = wl["cfg"]
    P, W, K = args.prompt or wl["prompt"], args.warmup, args.steps
    max_seq = max(P + wl["gen"], P + W + K)
    dist = None
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("LLMQ_THREADS", str(max(1, (os.cpu_count() or 1) // world)))
    m = make_model(lib, cfg, max_seq)
    t0 = time.time()
    if lib.q_llama_model_upload(C.byref(m)) != 0:
        raise RuntimeError(lib.q_llama_last_error_message().decode())
    log(f"uploaded in {time.time() - t0:.1f}s")
    kv = lib.q_llama_kv_create(C.byref(m))
    llmq.check(lib)

    # prompt, token by token through the reference-facing call (untimed)
    prompt = prompt_ids(cfg, P)
    nxt = -1
    for t in prompt:
        nxt = lib.q_llama_decode_step_argmax(C.byref(m), C.byref(kv), int(t), None)
    llmq.check(lib)

    # warm-up: W greedy steps chained on the device
    ids = (C.c_int * max(W, K, 1))()
    if lib.q_llama_generate(C.byref(m), C.byref(kv), nxt, W, ids) != 0:
        llmq.check(lib)
    start_len, start_tok = kv.len, ids[W - 1]

    # ---- timed region: K greedy steps, device-chained
    if dist is not None:
        dist.barrier()
    with ClockSampler(local) as clk:
        if lib.q_llama_generate(C.byref(m), C.byref(kv), start_tok, K, ids) != 0:
            llmq.check(lib)
        ms = float(lib.q_llama_last_step_ms())
    gen_ids = [ids[i] for i in range(K)]
    ms = max_over_ranks([ms], dist)[0]
    if dist is not None:
        dist.barrier()
    value = world * K / (ms / 1e3)

    # ---- e2e: the same K positions again through q_llama_decode_step
    kv.len = start_len
    logits = np.zeros((1, cfg["vocab"]), np.float32)
    lt = llmq.host_tensor(logits)
    tok, e2e_ids = start_tok, []
    t0 = time.perf_counter()
    for _ in range(K):
        lib.q_llama_decode_step(C.byref(m), C.byref(kv), tok, C.byref(lt))
        tok = int(np.argmax(logits[0]))
        e2e_ids.append(tok)
    e2e_s = time.perf_counter() - t0
    llmq.check(lib)
    e2e_value = world * K / max_over_ranks([e2e_s], dist)[0]

    # ---- the same K positions with the CLI's sampler settings (main.c:643-645),
    # drawn on the device inside each step's graph
    kv.len = start_len
    rng = lib.rng_create(1234)
    if lib.q_llama_generate_sample(C.byref(m), C.byref(kv), start_tok, K, 0.8, 40, 0.95, C.byref(rng), ids) != 0:
        llmq.check(lib)
    s_ms = float(lib.q_llama_last_step_ms())
    sampled = {"value": round(world * K / (s_ms / 1e3), 2), "unit": "tok/s", "ms_per_step": round(s_ms / K, 4),
               "api": "q_llama_generate_sample (temperature 0.8, top-k 40, top-p 0.95, seed 1234)",
               "sampler_ms_per_step": round((s_ms - ms) / K, 4)}

    # ---- one step replayed kernel by kernel (no graph, no overlap): where the time goes
    nk = int(lib.llmq_kernels_per_step(C.byref(m)))
    prof = np.zeros(nk, np.float32)
    kv.len = start_len
    if lib.llmq_step_profile(C.byref(m), C.byref(kv), start_tok, prof.ctypes.data_as(llmq.c_float_p), nk) != 0:
        llmq.check(lib)
    per_layer = (nk - 2) // cfg["n_layers"]
    names = ["qkv", "attn", "wo", "w13", "w2"] if per_layer == 5 else ["qkv", "attn_scores", "attn_pv", "wo", "w13", "w2"]
    step_profile = {n: round(float(prof[i:nk - 2:len(names)].sum()), 4) for i, n in enumerate(names)}
    step_profile.update(lm_head=round(float(prof[nk - 2]), 4), finish=round(float(prof[nk - 1]), 4),
                        total=round(float(prof.sum()), 4), unit="ms per step, kernels serialised")

    # ---- roofline of the GEMV kernel: per-kind CUDA-event timings
    kinds = [(0, cfg["n_layers"]), (1, cfg["n_layers"]), (2, cfg["n_layers"]), (3, cfg["n_layers"]), (4, 1)]
    g_bytes, g_ms, per_kind = 0.0, 0.0, {}
    for which, count in kinds:
        msl, by = C.c_float(), C.c_double()
        # one launch per layer (different weights each time), from one CUDA graph
        if lib.llmq_bench_gemv(C.byref(m), which, 0, cfg["n_layers"], C.byref(msl), C.byref(by)) != 0:
            llmq.check(lib)
        g_bytes += count * by.value
        g_ms += count * msl.value
        per_kind[["qkv", "wo", "w13", "w2", "lm_head"][which]] = {
            "ms": round(msl.value, 5), "GBps": round(by.value / msl.value / 1e6, 1)}
    msl, by = C.c_float(), C.c_double()
    if lib.llmq_bench_gemv(C.byref(m), 5, 0, cfg["n_layers"], C.byref(msl), C.byref(by)) != 0:
        llmq.check(lib)
    per_kind["attention"] = {"ms": round(msl.value, 5), "GBps": round(by.value / msl.value / 1e6, 1)}
    peaks = measured_peaks()
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = g_bytes / (g_ms / 1e3) / 1e9
    step_bytes = weight_bytes(cfg)
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4), "traffic": profiled_traffic(cfg),
                "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured)" if peaks else "fallback 6650 GB/s",
                "kernel": "k_gemv (int8 W8A8 GEMV, all five per-step shapes)",
                "per_kind": per_kind,
                "step_bytes": step_bytes,
                "step_frac": round(step_bytes / (ms / K / 1e3) / 1e9 / hbm_peak, 4)}

    # ---- CPU baseline: the reference's decode on the same model and cache
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        kv.len = start_len
        cpu = cpu_baseline(lib, m, kv, start_tok, gen_ids)

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms / K, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": bs1_config(args, wl, P, W, K, world),
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 16 + 4 * cfg["vocab"],
                "api": "q_llama_decode_step (host token, host f32 logits, host argmax)",
                "same_tokens_as_value_run": e2e_ids == gen_ids},
        "roofline": roofline,
        "cpu_baseline": cpu,
        "sampled_decode": sampled,
        "step_profile": step_profile,
        "gpu_launches": K * int(lib.llmq_kernels_per_step(C.byref(m))),
        "clocks": clk.summary(),
    }
    lib.llama_kv_free(C.byref(kv))

    # ---- N > 1: the same model and prompt as one tensor-parallel group
    if world > 1 and args.workload == "8b" and not args.no_tp_leg:
        line["tp"] = tp_leg(lib, m, cfg, prompt, W, K, gen_ids, rank, world, local, hbm_peak, dist)
    lib.q_llama_model_free(C.byref(m))

    # ---- one GPU: the other configs of the metric, as objects of the same line
    if world == 1 and args.workload == "8b" and not args.no_extra:
        line["bs64"] = bs64_leg(lib, args, hbm_peak, peaks)
        line["tiny"] = tiny_leg(lib, args)
        line["gemv_sweep"] = gemv_sweep(lib, [1, 8, 64, 256], hbm_peak, cpu=not args.no_cpu_baseline)
    if rank == 0:
        print(json.dumps(line), flush=True)


def tp_leg(lib, m, cfg, prompt, W, K, gen_ids, rank, world, local, hbm_peak, dist):
    """The bs1 workload on one tensor-parallel group of all N ranks: each rank
    cuts its shard of the same model (q_llama_model_shard), decodes the same
    prompt and warm-up, then K timed device-chained steps.  The greedy ids must
    equal this rank's 1-GPU run of the same positions (gen_ids).  The
    row-parallel products exchange their int32 partial sums over NVLink peer
    memory inside the GEMV; one NCCL max-reduce of the argmax key closes each
    step."""
    t0 = time.time()
    llmq.tp_bootstrap(lib, rank, world)
    sh = llmq.QLlamaModel()
    if lib.q_llama_model_shard(C.byref(m), rank, world, C.byref(sh)) != 0:
        llmq.check(lib)
    if lib.q_llama_model_upload(C.byref(sh)) != 0:
        llmq.check(lib)
    kv = lib.q_llama_kv_create(C.byref(sh))
    llmq.check(lib)
    nxt = -1
    for t in prompt:
        nxt = lib.q_llama_decode_step_argmax(C.byref(sh), C.byref(kv), int(t), None)
    llmq.check(lib)
    ids = (C.c_int * max(W, K, 1))()
    if lib.q_llama_generate(C.byref(sh), C.byref(kv), nxt, W, ids) != 0:
        llmq.check(lib)
    start_tok = ids[W - 1]
    log(f"rank {rank}: tensor-parallel shard ready in {time.time() - t0:.1f}s")
    dist.barrier()
    with ClockSampler(local) as clk:
        if lib.q_llama_generate(C.byref(sh), C.byref(kv), start_tok, K, ids) != 0:
            llmq.check(lib)
        ms = float(lib.q_llama_last_step_ms())
    tp_ids = [ids[i] for i in range(K)]
    mismatch = 0.0 if tp_ids == gen_ids else 1.0
    ms, mismatch = max_over_ranks([ms, mismatch], dist)
    per_rank_bytes = weight_bytes(cfg) / world
    achieved = per_rank_bytes / (ms / K / 1e3) / 1e9
    out = {"value": round(K / (ms / 1e3), 2), "unit": "tok/s", "ms_per_step": round(ms / K, 4), "group": world,
           "scaling": "strong", "steps": K,
           "greedy_ids_match_1gpu": mismatch == 0.0,
           "workload": "the bs1 workload (same model, prompt and positions) decoded by one tensor-parallel group",
           "exchange": "row-parallel Wo/W2: int32 partial sums and absmax over NVLink peer memory inside the GEMV "
                       "(bounded flag waits); argmax: NCCL max-reduce of the argmax key; all in the step's CUDA graph",
           "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                        "frac": round(achieved / hbm_peak, 4),
                        "kernel": "whole decode step per GPU (this rank's int8 weight shard read once)"},
           "gpu_launches": K * int(lib.llmq_kernels_per_step(C.byref(sh))),
           "clocks": clk.summary()}
    lib.llama_kv_free(C.byref(kv))
    lib.q_llama_model_free(C.byref(sh))
    dist.barrier()
    lib.q_llama_tp_shutdown()
    return out


def bs64_leg(lib, args, hbm_peak, peaks):
    """configs[3] on one GPU inside the default line: 64 sequences, each a
    2048-id prompt prefilled, then W warm-up and a bounded number of timed
    batched greedy decode steps (KV 2048 + W ..)."""
    wl = WORKLOADS["serve64"]
    cfg, B, P = wl["cfg"], wl["batch"], wl["prompt"]
    W, K = 3, 16
    m = make_model(lib, cfg, P + W + K)
    if lib.q_llama_model_upload(C.byref(m)) != 0:
        llmq.check(lib)
    r = serve_measure(lib, m, cfg, B, P, W, K, 0, None)
    lib.q_llama_model_free(C.byref(m))
    return serve_summary(r, cfg, B, P, W, K, 1, False, hbm_peak, peaks, wl)


def tiny_leg(lib, args):
    """configs[0] inside the default line: the tiny model, a 16-id prompt then
    240 greedy tokens chained on the GPU (us/token), the same 240 positions
    through q_llama_decode_step (e2e), and the reference's CPU decode of the
    same tokens on the same model (oracle/_ref)."""
    wl = WORKLOADS["tiny"]
    cfg, P, G = wl["cfg"], wl["prompt"], wl["gen"]
    m = make_model(lib, cfg, P + G)
    if lib.q_llama_model_upload(C.byref(m)) != 0:
        llmq.check(lib)
    kv = lib.q_llama_kv_create(C.byref(m))
    llmq.check(lib)
    prompt = prompt_ids(cfg, P)
    nxt = -1
    for t in prompt:
        nxt = lib.q_llama_decode_step_argmax(C.byref(m), C.byref(kv), int(t), None)
    llmq.check(lib)
    ids = (C.c_int * G)()
    # warm-up on the same positions, then the timed run
    if lib.q_llama_generate(C.byref(m), C.byref(kv), nxt, G, ids) != 0:
        llmq.check(lib)
    kv.len = P
    if lib.q_llama_generate(C.byref(m), C.byref(kv), nxt, G, ids) != 0:
        llmq.check(lib)
    ms = float(lib.q_llama_last_step_ms())
    gen = [ids[i] for i in range(G)]
    kv.len = P
    logits = np.zeros((1, cfg["vocab"]), np.float32)
    lt = llmq.host_tensor(logits)
    tok = nxt
    t0 = time.perf_counter()
    for _ in range(G):
        lib.q_llama_decode_step(C.byref(m), C.byref(kv), tok, C.byref(lt))
        tok = int(np.argmax(logits[0]))
    e2e_s = time.perf_counter() - t0
    llmq.check(lib)
    out = {"value": round(G / (ms / 1e3), 1), "unit": "tok/s", "us_per_token": round(ms * 1e3 / G, 2),
           "steps": G, "prompt": P, "workload": wl["name"],
           "e2e": {"value": round(G / e2e_s, 1), "unit": "tok/s", "us_per_token": round(e2e_s * 1e6 / G, 2),
                   "api": "q_llama_decode_step (host token, host f32 logits, host argmax)"},
           "roofline": "latency-bound: 14.5 MB of weights fit in L2; no HBM fraction is meaningful"}
    if not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        ref = oracle.load_reference()
        if ref is not None:
            rkv = ref.q_llama_kv_create(C.byref(m))
            for t in prompt:
                ref.q_llama_decode_step(C.byref(m), C.byref(rkv), int(t), C.byref(lt))
            tok, ref_ids = nxt, []
            t0 = time.perf_counter()
            for _ in range(G):
                ref.q_llama_decode_step(C.byref(m), C.byref(rkv), tok, C.byref(lt))
                tok = int(np.argmax(logits[0]))
                ref_ids.append(tok)
            dt = time.perf_counter() - t0
            ref.llama_kv_free(C.byref(rkv))
            out["cpu_baseline"] = {"value": round(G / dt, 1), "unit": "tok/s", "us_per_token": round(dt * 1e6 / G, 2),
                                   "cores": min(os.cpu_count() or 1, 64), "kind": "reference",
                                   "sample": f"the same {G} greedy tokens after the same {P}-id prompt",
                                   "greedy_ids_match_gpu": ref_ids == gen}
    lib.llama_kv_free(C.byref(kv))
    lib.q_llama_model_free(C.byref(m))
    return out


def measured_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        return {}


def run_f32(args, rank, world):
    """The fp32 (LLMA) path: llama_decode_step on a dequantised 8B-shaped model.
    A step is one token; value from K device-chained steps (llama_generate),
    e2e through llama_decode_step with the logits row copied to the host."""
    lib = llmq.load()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if lib.q_llama_set_device(local) != 0:
        raise RuntimeError(lib.q_llama_last_error_message().decode())
    wl = WORKLOADS[args.workload]
    cfg = wl["cfg"]
    P, W, K = args.prompt or wl["prompt"], args.warmup, args.steps
    c = llmq.config(max_seq=P + W + 2 * K + 8, **cfg)
    m = llmq.LlamaModel()
    t0 = time.time()
    if lib.llmq_synth_model_f32(C.byref(c), SEED_WEIGHTS, 0.02, 0, C.byref(m)) != 0:
        llmq.check(lib)
    log(f"fp32 synthetic model built in {time.time() - t0:.1f}s")
    t0 = time.time()
    if lib.llmq_llama_model_upload(C.byref(m)) != 0:
        llmq.check(lib)
    log(f"uploaded in {time.time() - t0:.1f}s")
    kv = lib.llama_kv_create(C.byref(m))
    llmq.check(lib)
    nxt = -1
    for t in prompt_ids(cfg, P):
        nxt = lib.llama_decode_step_argmax(C.byref(m), C.byref(kv), int(t), None)
    llmq.check(lib)
    ids = (C.c_int * max(W, K))()
    if lib.llama_generate(C.byref(m), C.byref(kv), nxt, W, ids) != 0:
        llmq.check(lib)
    start_len, start_tok = kv.len, ids[W - 1]
    with ClockSampler(local) as clk:
        if lib.llama_generate(C.byref(m), C.byref(kv), start_tok, K, ids) != 0:
            llmq.check(lib)
        ms = float(lib.q_llama_last_step_ms())
    gen_ids = [ids[i] for i in range(K)]
    value = world * K / (ms / 1e3)
    kv.len = start_len
    logits = np.zeros((1, cfg["vocab"]), np.float32)
    lt = llmq.host_tensor(logits)
    tok, e2e_ids = start_tok, []
    t0 = time.perf_counter()
    for _ in range(K):
        lib.llama_decode_step(C.byref(m), C.byref(kv), tok, C.byref(lt))
        tok = int(np.argmax(logits[0]))
        e2e_ids.append(tok)
    e2e_s = time.perf_counter() - t0
    llmq.check(lib)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    step_bytes = 4 * weight_bytes(cfg)
    achieved = step_bytes / (ms / K / 1e3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = f32_cpu_baseline(m, cfg)
    line = {
        "metric": "fp32-weight decode tok/s (bs1)", "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(ms / K, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl["name"], "kv_len_start": start_len, "kv_len_end": start_len + K, "prompt": P,
                   "parallelism": "single GPU" if world == 1 else f"{world} independent replicas",
                   "l2": f"inputs larger than L2: {step_bytes / 1e9:.1f} GB of fp32 weights streamed per step"},
        "e2e": {"value": round(world * K / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 16 + 4 * cfg["vocab"], "api": "llama_decode_step (host logits, host argmax)",
                "same_tokens_as_value_run": e2e_ids == gen_ids},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": None,
                     "kernel": "whole step: fp32 weight bytes per step / step time (k_gemv_f32 dominates)",
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured)" if peaks else "fallback 6650 GB/s"},
        "cpu_baseline": cpu,
        # per step: QKV, attention (1 or 2), Wo, W1|W3, W2 per layer; lm-head, finish
        "gpu_launches": K * ((4 + int(lib.llmq_attention_launches(cfg["n_heads"], cfg["n_kv"], cfg["head_dim"],
                                                                  int(c.max_seq)))) * cfg["n_layers"] + 2),
        "clocks": clk.summary(),
    }
    lib.llama_kv_free(C.byref(kv))
    lib.llmq_llama_model_free(C.byref(m))
    if rank == 0:
        print(json.dumps(line), flush=True)


def f32_cpu_baseline(m, cfg):
    """The reference's own llama_decode_step (oracle/_ref) on the same fp32
    model, from an empty cache, for about 10 s on the host cores."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    ref = oracle.load_reference()
    if ref is None:
        return None
    kv = ref.llama_kv_create(C.byref(m))
    row = np.zeros((1, cfg["vocab"]), np.float32)
    t = llmq.host_tensor(row)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 10.0 and n < 64:
        ref.llama_decode_step(C.byref(m), C.byref(kv), int(n * 7 % cfg["vocab"]), C.byref(t))
        n += 1
    dt = time.perf_counter() - t0
    ref.llama_kv_free(C.byref(kv))
    # matrix.c's matmul threads over output rows (parallel_for(M)); a decode
    # step has one row, so the reference runs it on one core
    return {"value": round(n / dt, 4), "unit": "tok/s", "cores": 1, "kind": "reference",
            "sample": f"{n} fp32 decode steps of the same model at positions 0..{n - 1}"}


def serve_measure(lib, m, cfg, B, P, W, K, local, dist):
    """B sequences each prefilled with its own P-id prompt
    (q_llama_prefill_argmax, one sequence per call; the GEMMs see up to 1024
    rows), then W warm-up and K timed batched greedy decode steps
    (q_llama_decode_batch_argmax, one row per sequence).  Returns the
    device-timed and wall-clock figures (max over ranks)."""
    kvs = []
    for _ in range(B):
        kvs.append(lib.q_llama_kv_create(C.byref(m)))
        llmq.check(lib)
    rng = np.random.default_rng(SEED_PROMPT)
    prompts = rng.integers(0, cfg["vocab"], size=(B, P)).astype(np.int32)
    pre_ms, nxt = 0.0, []
    t0 = time.perf_counter()
    for b in range(B):
        tok = lib.q_llama_prefill_argmax(C.byref(m), C.byref(kvs[b]), prompts[b].ctypes.data_as(llmq.c_int_p), P,
                                         None)
        if tok < 0:
            llmq.check(lib)
        pre_ms += float(lib.q_llama_last_step_ms())
        nxt.append(tok)
    pre_wall = time.perf_counter() - t0
    kvp = llmq.kv_pointers(kvs)
    out = (C.c_int * B)()

    def step(tokens):
        rc = lib.q_llama_decode_batch_argmax(C.byref(m), kvp, llmq.int_array(tokens), B, out)
        if rc != 0:
            llmq.check(lib)
        return [out[i] for i in range(B)], float(lib.q_llama_last_step_ms())

    for _ in range(W):
        nxt, _ = step(nxt)
    if dist is not None:
        dist.barrier()
    dev_ms, launches = 0.0, 0
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        for _ in range(K):
            nxt, ms = step(nxt)
            dev_ms += ms
            launches += int(lib.llmq_last_launches())
        wall = time.perf_counter() - t0
    dev_ms, wall, pre_ms = max_over_ranks([dev_ms, wall, pre_ms], dist)
    for kv in kvs:
        lib.llama_kv_free(C.byref(kv))
    return {"dev_ms": dev_ms, "wall": wall, "pre_ms": pre_ms, "pre_wall": pre_wall, "launches": launches,
            "clocks": clk.summary()}


def serve_summary(r, cfg, B, P, W, K, groups, tp, hbm_peak, peaks, wl, world=1):
    """The decode, prefill, e2e and roofline figures of one serve_measure."""
    kvd = cfg["n_kv"] * cfg["head_dim"]
    mean_pos = P + W + (K - 1) / 2.0
    kv_bytes = B * cfg["n_layers"] * 2 * (mean_pos + 1) * kvd * 4
    step_bytes = weight_bytes(cfg) + kv_bytes
    if tp:  # per GPU: its shard of the weights and of the KV heads
        step_bytes /= world
    achieved = step_bytes / (r["dev_ms"] / K / 1e3) / 1e9
    # prefill: int8 tensor-core products (every layer's weights for every prompt
    # row, the lm-head for each prompt's last row) plus the attention's
    # products (q.k and p.v over the causal prefix)
    lm = cfg["d_model"] * cfg["vocab"]
    w_ops = 2.0 * (weight_bytes(cfg) - lm) * B * P + 2.0 * lm * B
    attn_ops = 2.0 * 2.0 * cfg["n_layers"] * cfg["n_heads"] * cfg["head_dim"] * B * P * (P + 1) / 2.0
    pre_tops = (w_ops + attn_ops) / (r["pre_ms"] / 1e3) / 1e12
    if tp:
        pre_tops /= world
    bf16 = float(peaks.get("bf16_tflops", 1590.0))
    return {
        "value": round(groups * B * K / (r["dev_ms"] / 1e3), 1), "unit": "tok/s",
        "ms_per_step": round(r["dev_ms"] / K, 4), "steps": K, "warmup": W, "batch": B, "prompt": P,
        "kv_len_start": P + W, "kv_len_end": P + W + K, "workload": wl["name"],
        "prefill": {"tok_per_s": round(groups * B * P / (r["pre_ms"] / 1e3), 1), "gpu_ms": round(r["pre_ms"], 1),
                    "wall_s": round(r["pre_wall"], 2), "api": "q_llama_prefill_argmax, one sequence per call",
                    "tensor": {"bound": "tensor", "achieved": round(pre_tops, 1), "unit": "TOP/s (int8)",
                               "peak": bf16, "frac": round(pre_tops / bf16, 4),
                               "peak_source": "MEASURED_PEAKS.json bf16_tflops (measured bf16 burst; the int8 "
                                              "dense rate is nominally twice it)" if peaks else "fallback 1590",
                               "algorithmic_ops": w_ops + attn_ops}},
        "e2e": {"value": round(groups * B * K / r["wall"], 1), "unit": "tok/s", "h2d_bytes_per_step": B * (4 + 32),
                "d2h_bytes_per_step": B * 4 + 4,
                "api": "q_llama_decode_batch_argmax (host ids in and out, one call per step)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": None,
                     "kernel": "whole batched step (weights + f32 KV rows read once)",
                     "step_bytes": int(step_bytes)},
        "gpu_launches": r["launches"],
        "clocks": r["clocks"],
    }


def run_serve(args, rank, world):
    """configs[3] (and configs[4] at batch 32): a step is one batched decode
    step (B tokens)."""
    lib = llmq.load()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if lib.q_llama_set_device(local) != 0:
        raise RuntimeError(lib.q_llama_last_error_message().decode())
    wl = WORKLOADS[args.workload]
    cfg = wl["cfg"]
    B, P, W, K = wl["batch"], args.prompt or wl["prompt"], args.warmup, args.steps
    max_seq = P + W + K
    tp = bool(wl.get("tp")) and world > 1
    dist = None
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("LLMQ_THREADS", str(max(1, (os.cpu_count() or 1) // world)))
    if tp:  # one tensor-parallel group over all ranks; each rank builds its shard
        llmq.tp_bootstrap(lib, rank, world)
    if tp or wl.get("fast"):
        c = llmq.config(max_seq=max_seq, **cfg)
        m = llmq.QLlamaModel()
        r_, w_ = (rank, world) if tp else (0, 1)
        if wl.get("fast"):
            rc = lib.llmq_synth_model_fast_shard(C.byref(c), SEED_WEIGHTS, r_, w_, C.byref(m))
        else:
            rc = lib.llmq_synth_model_shard(C.byref(c), SEED_WEIGHTS, 0.02, 0, r_, w_, C.byref(m))
        if rc != 0:
            llmq.check(lib)
    else:
        m = make_model(lib, cfg, max_seq)
    if lib.q_llama_model_upload(C.byref(m)) != 0:
        raise RuntimeError(lib.q_llama_last_error_message().decode())
    r = serve_measure(lib, m, cfg, B, P, W, K, local, dist)
    groups = 1 if tp else world  # replicas each serve their own B sequences
    peaks = measured_peaks()
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    s = serve_summary(r, cfg, B, P, W, K, groups, tp, hbm_peak, peaks, wl, world)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not wl.get("fast"):
        cpu = serve_cpu_baseline(lib, m, cfg)
    line = {
        "metric": f"int8-weight decode tok/s (bs{B})", "value": s["value"], "unit": "tok/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": s["ms_per_step"], "higher_is_better": True,
        "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded uniform int8 codes, per-column scales)" if wl.get("fast") else "synthetic",
        "config": {"workload": wl["name"], "model": f"{args.workload}-shaped synthetic, seed {SEED_WEIGHTS}",
                   "global_batch": B * groups, "prompt": P, "kv_len_start": P + W, "kv_len_end": P + W + K,
                   "parallelism": f"tp{world}" if tp else "single GPU per replica",
                   "l2": f"inputs larger than L2: {s['roofline']['step_bytes'] / 1e9:.1f} GB of weights and KV "
                         f"per GPU per step"},
        "prefill": s["prefill"], "e2e": s["e2e"], "roofline": s["roofline"], "cpu_baseline": cpu,
        "gpu_launches": s["gpu_launches"], "clocks": s["clocks"],
    }
    lib.q_llama_model_free(C.byref(m))
    if tp:
        dist.barrier()
        lib.q_llama_tp_shutdown()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_tp(args, rank, world):
    """one sequence decoded by a tensor-parallel group of all N
    GPUs (N = 1: the whole model on one GPU).  Weights: the fast seeded
    generator (uniform int8 codes, per-column scales), shard per rank.  A step
    is one token; value = tokens/s of the sequence (strong scaling)."""
    lib = llmq.load()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if lib.q_llama_set_device(local) != 0:
        raise RuntimeError(lib.q_llama_last_error_message().decode())
    wl = WORKLOADS[args.workload]
    cfg = wl["cfg"]
    P, W, K = args.prompt or wl["prompt"], args.warmup, args.steps
    max_seq = P + W + K
    os.environ.setdefault("LLMQ_THREADS", str(max(1, (os.cpu_count() or 1) // world)))
    dist = None
    if world > 1:
        import torch
        import torch.distributed as dist
        llmq.tp_bootstrap(lib, rank, world)
    c = llmq.config(max_seq=max_seq, **cfg)
    m = llmq.QLlamaModel()
    t0 = time.time()
    if lib.llmq_synth_model_fast_shard(C.byref(c), SEED_WEIGHTS, rank, world, C.byref(m)) != 0:
        llmq.check(lib)
    log(f"rank {rank}: shard built in {time.time() - t0:.1f}s")
    t0 = time.time()
    if lib.q_llama_model_upload(C.byref(m)) != 0:
        llmq.check(lib)
    log(f"rank {rank}: uploaded in {time.time() - t0:.1f}s")
    kv = lib.q_llama_kv_create(C.byref(m))
    llmq.check(lib)
    nxt = -1
    for t in prompt_ids(cfg, P):
        nxt = lib.q_llama_decode_step_argmax(C.byref(m), C.byref(kv), int(t), None)
    llmq.check(lib)
    ids = (C.c_int * max(W, K, 1))()
    if lib.q_llama_generate(C.byref(m), C.byref(kv), nxt, W, ids) != 0:
        llmq.check(lib)
    start_len, start_tok = kv.len, ids[W - 1]

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if dist is not None:
        dist.barrier()
    with ClockSampler(local) as clk:
        if lib.q_llama_generate(C.byref(m), C.byref(kv), start_tok, K, ids) != 0:
            llmq.check(lib)
        ms = max_over_ranks(float(lib.q_llama_last_step_ms()))
    gen_ids = [ids[i] for i in range(K)]
    value = K / (ms / 1e3)
    # e2e: the same positions through q_llama_decode_step (host token in, whole
    # logits row out on every rank, host argmax)
    kv.len = start_len
    logits = np.zeros((1, cfg["vocab"]), np.float32)
    lt = llmq.host_tensor(logits)
    tok, e2e_ids = start_tok, []
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        lib.q_llama_decode_step(C.byref(m), C.byref(kv), tok, C.byref(lt))
        tok = int(np.argmax(logits[0]))
        e2e_ids.append(tok)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    llmq.check(lib)
    hbm_peak = hbm_peak_gbs()
    per_rank_bytes = weight_bytes(cfg) / world
    achieved = per_rank_bytes / (ms / K / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms / K, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic (seeded uniform int8 codes, per-column scales)",
        "config": {"workload": wl["name"], "model": f"70b-shaped synthetic, seed {SEED_WEIGHTS}",
                   "global_batch": 1, "prompt": P, "kv_len_start": start_len, "kv_len_end": start_len + K,
                   "parallelism": f"tp{world}",
                   "l2": f"inputs larger than L2: {per_rank_bytes / 1e9:.2f} GB of int8 weights per GPU per step"},
        "e2e": {"value": round(K / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 16 + 4 * cfg["vocab"],
                "api": "q_llama_decode_step on every rank (host token, whole f32 logits row, host argmax)",
                "same_tokens_as_value_run": e2e_ids == gen_ids},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": None,
                     "kernel": "whole decode step per GPU (this rank's int8 weights read once)"},
        "cpu_baseline": None,
        "gpu_launches": K * int(lib.llmq_kernels_per_step(C.byref(m))),
        "clocks": clk.summary(),
    }
    lib.llama_kv_free(C.byref(kv))
    lib.q_llama_model_free(C.byref(m))
    if world > 1:
        dist.barrier()
        lib.q_llama_tp_shutdown()
    if rank == 0:
        print(json.dumps(line), flush=True)


def serve_cpu_baseline(m, cfg, P):
    """The reference's q_llama_decode_step on the host cores for one sequence
    whose first P cache rows are seeded values (as in the reference arm).  The
    reference has no batch entry point: B sequences cost B times one, so its
    batch-B tokens/s equals this single-sequence rate."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    cores = os.cpu_count() or 1
    os.environ["TF_THREADS"] = str(min(cores, 64))
    ref = oracle.load_reference()
    if ref is None:
        return None
    kv = ref.q_llama_kv_create(C.byref(m))
    seed_prompt_rows(kv, P)
    logits = np.zeros((1, m.vocab), np.float32)
    lt = llmq.host_tensor(logits)
    tok, n, t_total = 1, 0, 0.0
    while n < 32 and t_total < 15.0 and kv.len < kv.max_seq:
        t0 = time.perf_counter()
        ref.q_llama_decode_step(C.byref(m), C.byref(kv), tok, C.byref(lt))
        t_total += time.perf_counter() - t0
        tok = int(np.argmax(logits[0]))
        n += 1
    ref.llama_kv_free(C.byref(kv))
    return {"value": round(n / t_total, 4), "unit": "tok/s", "cores": min(cores, 64), "kind": "reference",
            "sample": f"{n} single-sequence decode steps at positions {P}..{P + n - 1} (prompt cache rows seeded; "
                      f"the reference decodes a batch one sequence at a time)"}


def seed_prompt_rows(kv, P):
    """Fills cache rows [0, P) of a reference LlamaKV with seeded N(0, 1)
    values and sets kv.len = P (in place of decoding a long prompt on the CPU)."""
    rng = np.random.default_rng(SEED_PROMPT)
    kvd = kv.kv_dim
    for l in range(kv.n_layers):
        for arr in (kv.k, kv.v):
            a = np.ctypeslib.as_array(arr[l], shape=(kv.max_seq * kvd,))
            a[: P * kvd] = rng.standard_normal(P * kvd).astype(np.float32)
    kv.len = P


SWEEP_SHAPES = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]  # (out, in)


def gemv_sweep(lib, Ms, hbm_peak, iters=20, cpu=False, cpu_budget_s=25.0):
    """isolated int8 products on uniform int8 codes with scales in
    [1e-3, 1e-2), device-resident A; GB/s of algorithmic bytes and % of HBM.
    With cpu=True the reference's own qmatmul (oracle/_ref, all host cores)
    multiplies the same W by N(0, 1) activations once per cell, beside it
    (cells after the first ~25 s of CPU time are left out: null)."""
    ref = None
    if cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        os.environ["TF_THREADS"] = str(min(os.cpu_count() or 1, 64))
        ref = oracle.load_reference()
    cpu_spent, rows = 0.0, []
    g = np.random.default_rng(SEED_PROMPT)
    for out_f, in_f in SWEEP_SHAPES:
        t = lib.qtensor_create(in_f, out_f)  # reference layout: rows = in, cols = out
        lib.llmq_synth_qtensor(C.byref(t), 4321)
        for M in Ms:
            ms = C.c_float()
            if lib.llmq_bench_qmatmul(C.byref(t), M, iters, C.byref(ms)) != 0:
                llmq.check(lib)
            K, N = in_f, out_f
            by = K * N + 4 * N + 4 * M * K + 4 * M * N
            gbs = by / (ms.value / 1e3) / 1e9
            row = {"out_x_in": f"{out_f}x{in_f}", "M": M, "us": round(ms.value * 1e3, 2),
                   "GBps": round(gbs, 1), "hbm_frac": round(gbs / hbm_peak, 3),
                   "TOPS": round(2.0 * M * K * N / (ms.value / 1e3) / 1e12, 1)}
            if ref is not None:
                row["cpu_us"] = None
                if cpu_spent < cpu_budget_s:
                    A = g.standard_normal((M, K)).astype(np.float32)
                    Cm = np.zeros((M, N), np.float32)
                    ta, tc = llmq.host_tensor(A), llmq.host_tensor(Cm)
                    if not rows:  # start the reference's thread pool outside the timing
                        ref.qmatmul(C.byref(ta), C.byref(t), C.byref(tc))
                    t0 = time.perf_counter()
                    ref.qmatmul(C.byref(ta), C.byref(t), C.byref(tc))
                    dt = time.perf_counter() - t0
                    cpu_spent += dt
                    row["cpu_us"] = round(dt * 1e6, 1)
                    row["gpu_vs_cpu"] = round(dt * 1e3 / ms.value, 1)
            rows.append(row)
        lib.qtensor_free(C.byref(t))
    return rows


def run_sweep(args):
    lib = llmq.load()
    if lib.q_llama_set_device(int(os.environ.get("LOCAL_RANK", "0"))) != 0:
        raise RuntimeError(lib.q_llama_last_error_message().decode())
    peak = hbm_peak_gbs()
    rows = gemv_sweep(lib, [1, 8, 64, 256], peak, cpu=not args.no_cpu_baseline)
    m1 = sorted(r["GBps"] for r in rows if r["M"] == 1)
    print(json.dumps({"metric": "int8 W8A8 matvec/matmul GB/s (configs[1] sweep, M=1 median)",
                      "value": m1[len(m1) // 2], "unit": "GB/s", "n_gpus": 1, "higher_is_better": True,
                      "dtype": "int8", "data": "synthetic", "hbm_peak_gbs": peak,
                      "config": {"workload": "isolated int8 per-channel products, shapes (out x in) "
                                             + ", ".join(f"{o}x{i}" for o, i in SWEEP_SHAPES)
                                             + "; M = 1, 8, 64, 256",
                                 "path": "k_gemv (dp4a) for M <= 8, k_tc_gemm (tcgen05.mma.kind::i8) above",
                                 "cpu": "cpu_us: the reference's qmatmul (oracle/_ref), all host cores, one call"},
                      "sweep": rows}), flush=True)


def hbm_peak_gbs():
    try:
        return float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def profiled_traffic(cfg):
    """Mean DRAM bytes per k_gemv launch of one decode step, from the per-kind
    ncu figures committed in profiles/k_gemv_8b_decode.md (captured on the
    8B layer shapes; the step has n_layers launches of each layer kind and one
    lm_head).  None for other shapes."""
    if (cfg["d_model"], cfg["d_ff"], cfg["vocab"], cfg["n_heads"], cfg["n_kv"]) != (4096, 14336, 128256, 32, 8):
        return None
    per = {}
    try:
        for ln in open(os.path.join(ROOT, "profiles", "k_gemv_8b_decode.md")):
            if ln.startswith("traffic_bytes "):
                k, v = ln[len("traffic_bytes "):].split(":", 1)
                per[k.strip()] = float(v)
    except (OSError, ValueError):
        return None
    if not {"qkv", "wo", "w13", "w2", "lm_head"} <= per.keys():
        return None
    L = cfg["n_layers"]
    return round((L * (per["qkv"] + per["wo"] + per["w13"] + per["w2"]) + per["lm_head"]) / (4 * L + 1))


def cpu_baseline(lib, m, kv, start_tok, gen_ids):
    """Times the reference's q_llama_decode_step on the host cores, continuing
    from the GPU-built cache (copied to the host arrays): a bounded sample of the
    same decode positions.  Also checks its logits equal ours bit for bit."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    cores = os.cpu_count() or 1
    os.environ["TF_THREADS"] = str(min(cores, 64))
    ref = oracle.load_reference()
    kind = "reference"
    if ref is None:
        return None
    if lib.q_llama_kv_sync_host(C.byref(m), C.byref(kv)) != 0:
        llmq.check(lib)
    vocab = m.vocab
    ref_logits = np.zeros((1, vocab), np.float32)
    rt = llmq.host_tensor(ref_logits)
    tok, n, t_total, match = start_tok, 0, 0.0, True
    budget = 15.0
    while n < len(gen_ids) and n < 64 and t_total < budget:
        t0 = time.perf_counter()
        ref.q_llama_decode_step(C.byref(m), C.byref(kv), tok, C.byref(rt))
        t_total += time.perf_counter() - t0
        tok = int(np.argmax(ref_logits[0]))
        match &= tok == gen_ids[n]
        n += 1
    return {"value": round(n / t_total, 4), "unit": "tok/s", "cores": min(cores, 64), "kind": kind,
            "sample": f"{n} decode steps of the same model at positions {kv.len - n}..{kv.len - 1}, "
                      f"continuing the GPU-built KV cache copied to host memory",
            "greedy_ids_match_gpu": bool(match)}


# ----------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    """The reference's own CPU decode (oracle/_ref: quant.c, matrix.c, llama.c
    ... compiled unchanged, all host threads) on our arm's config, metric and
    unit.  Its model comes from oracle/_build/libsynth.so (the same seeded
    generator built on its own), so no library of ours is mapped."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    cores = os.cpu_count() or 1
    os.environ["TF_THREADS"] = str(min(cores, 64))
    ref = oracle.load_reference()
    wl = WORKLOADS[args.workload]
    cfg = wl["cfg"]
    if wl.get("tp") or "batch" in wl or wl.get("f32"):
        print(json.dumps({"impl": "reference", "unavailable": f"workload {args.workload}: the reference CPU arm runs "
                                                              "the int8 single-sequence workloads (8b, 8b2, tiny)"}),
              flush=True)
        return
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref was not built from the reference "
                                                            "sources (make -C oracle REF=<reference checkout>)"}),
              flush=True)
        return
    synth = oracle.load_synth()
    P, W, K = args.prompt or wl["prompt"], args.warmup, args.steps
    max_seq = max(P + wl["gen"], P + W + K)
    c = llmq.config(max_seq=max_seq, **cfg)
    m = llmq.QLlamaModel()
    t0 = time.time()
    if synth.llmq_synth_model(C.byref(c), SEED_WEIGHTS, 0.02, 0, C.byref(m)) != 0:
        raise RuntimeError("synthetic model generation failed")
    log(f"synthetic model built in {time.time() - t0:.1f}s")
    kv = ref.q_llama_kv_create(C.byref(m))
    seed_prompt_rows(kv, P)
    logits = np.zeros((1, cfg["vocab"]), np.float32)
    lt = llmq.host_tensor(logits)
    tok = int(prompt_ids(cfg, P)[-1])
    for _ in range(W):
        ref.q_llama_decode_step(C.byref(m), C.byref(kv), tok, C.byref(lt))
        tok = int(np.argmax(logits[0]))
    t0 = time.perf_counter()
    for _ in range(K):
        ref.q_llama_decode_step(C.byref(m), C.byref(kv), tok, C.byref(lt))
        tok = int(np.argmax(logits[0]))
    dt = time.perf_counter() - t0
    value = K / dt
    line = {"metric": METRIC, "value": round(value, 4), "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(dt / K * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
            "config": bs1_config(args, wl, P, W, K, world),
            "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": min(cores, 64),
                             "kind": "reference",
                             "sample": f"{K} decode steps at positions {P + W}..{P + W + K - 1} by the reference's "
                                       f"CPU thread pool (TF_THREADS={min(cores, 64)}); prompt cache rows seeded"},
            "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    ref.llama_kv_free(C.byref(kv))
    ref.q_llama_model_free(C.byref(m))
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default 240; serve64: 112)")
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["sweep"], default="8b")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prompt", type=int, default=0, help="override the prompt length (profiling runs)")
    ap.add_argument("--no-extra", action="store_true",
                    help="default workload: leave out the bs64, tiny and gemv_sweep objects")
    ap.add_argument("--no-tp-leg", action="store_true",
                    help="default workload at N > 1: leave out the tensor-parallel leg")
    args = ap.parse_args()
    if args.steps is None:
        wl = WORKLOADS.get(args.workload, {})
        args.steps = wl["gen"] - args.warmup if "batch" in wl else 240
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    try:
        if args.workload == "sweep":
            if rank == 0 and args.impl == "ours":
                run_sweep(args)
        elif args.impl == "reference":
            run_reference(args, rank, world)
        elif "batch" in WORKLOADS[args.workload]:
            run_serve(args, rank, world)
        elif WORKLOADS[args.workload].get("tp"):
            run_tp(args, rank, world)
        elif WORKLOADS[args.workload].get("f32"):
            run_f32(args, rank, world)
        else:
            run_ours(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
