"""Tensor parallelism on 2 GPUs: every rank holds its shard (llmq_synth_model_shard)
and the group decodes as one model; logits and greedy ids must equal the
oracle's single-sequence decode of the whole model bit for bit
(tests/tp_worker.py does the work, one process per GPU)."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def gpu_count() -> int:
    import torch
    return torch.cuda.device_count()


def test_tp2_decode_matches_oracle(tmp_path):
    if gpu_count() < 2:
        pytest.skip("tensor parallelism needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = ["timeout", "-k", "30", "900", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(HERE, "tp_worker.py"), str(tmp_path)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, (r.stdout[-4000:], r.stderr[-4000:])
    verdicts = json.load(open(tmp_path / "tp.json"))
    assert verdicts and all(verdicts.values()), verdicts
