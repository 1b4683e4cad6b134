"""bench.py's driver contract, on the CPU: the reference arm (the reference's
own CPU decode, oracle/_ref) prints one JSON line with the contract's keys,
also under torchrun with two ranks (rank 0 alone runs and prints), and
warm-up below 3 steps is refused."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BENCH = os.path.join(ROOT, "bench.py")
ARGS = ["--impl", "reference", "--workload", "tiny", "--steps", "2", "--warmup", "3"]


def json_lines(out: str) -> list[dict]:
    return [json.loads(line) for line in out.splitlines() if line.startswith("{")]


@pytest.fixture(scope="module")
def have_reference():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    if oracle.load_reference() is None:
        pytest.skip("reference build (oracle/_ref) not available")


def test_reference_arm_json_line(lib, have_reference):
    r = subprocess.run([sys.executable, BENCH] + ARGS, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1, r.stdout
    d = lines[0]
    assert d["impl"] == "reference"
    assert d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["dtype"] == "int8" and d["data"] == "synthetic"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_two_ranks_prints_once(lib, have_reference):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), BENCH] + ARGS
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1 and lines[0]["impl"] == "reference", r.stdout


def test_warmup_below_three_is_refused():
    r = subprocess.run([sys.executable, BENCH, "--impl", "reference", "--workload", "tiny", "--steps", "2",
                        "--warmup", "2"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode != 0 and "warmup" in r.stderr


def test_reference_arm_maps_no_library_of_ours(have_reference):
    """The reference arm builds its inputs with oracle/_build/libsynth.so and
    runs oracle/_ref alone: libllmq_cuda.so is never mapped into its process."""
    code = ("import runpy, sys\n"
            f"sys.argv = ['bench.py'] + {ARGS!r}\n"
            f"runpy.run_path({BENCH!r}, run_name='__main__')\n"
            "maps = open('/proc/self/maps').read()\n"
            "print('MAPPED', 'libllmq_cuda' in maps, 'libllmq_ref' in maps)\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "MAPPED False True" in r.stdout


def test_both_arms_print_the_same_config():
    """Both arms take their batch-1 `config` from one function."""
    sys.path.insert(0, ROOT)
    import argparse

    import bench
    args = argparse.Namespace(workload="8b", prompt=0)
    wl = bench.WORKLOADS["8b"]
    a = bench.bs1_config(args, wl, 512, 5, 20, 1)
    assert a == bench.bs1_config(args, wl, 512, 5, 20, 1)
    assert a["kv_len_start"] == 517 and a["kv_len_end"] == 537 and "seeded" in a["prompt_cache"]
    src = open(BENCH).read()
    assert src.count('"config": bs1_config(args, wl, P, W, K, world)') == 2
