"""Tensor parallelism on 2, 4 and 8 GPUs (as many as the machine has): every
rank holds its shard (llmq_synth_model_shard)
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


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decode_matches_oracle(tmp_path, world):
    if gpu_count() < world:
        pytest.skip(f"tensor parallelism over {world} ranks needs {world} GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = ["timeout", "-k", "30", "900", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(HERE, "tp_worker.py"), str(tmp_path)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, (r.stdout[-4000:], r.stderr[-4000:])
    verdicts = json.load(open(tmp_path / "tp.json"))
    assert verdicts and all(verdicts.values()), verdicts
