"""GPU: the link-level drop-in.  tests/link_check.c, compiled against the
reference's own headers and linked against libllmq_cuda.so alone (built by
__graft_entry__.build() or `make -C tests REF=<reference checkout>`), runs the
int8 half of the reference's selftest part [21] through this library; its
logits rows must equal, bit for bit, the rows the reference produced for the
same model (tests/golden/selftest21.*)."""
from __future__ import annotations

import os
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, ROOT, reference_dir

pytestmark = pytest.mark.gpu


def test_link_check_runs_selftest21_bit_exact(tmp_path):
    exe = os.path.join(ROOT, "tests", "_build", "link_check")
    ref = reference_dir()
    if ref is not None:
        subprocess.run(["make", "-C", os.path.join(ROOT, "tests"), f"REF={ref}"], check=True, capture_output=True)
    if not os.access(exe, os.X_OK):
        pytest.skip("link_check was not built (needs the reference headers at build time)")
    out = tmp_path / "logits.f32"
    env = dict(os.environ, LD_LIBRARY_PATH=os.path.join(ROOT, "llm-project_b200", "lib"))
    r = subprocess.run([exe, os.path.join(GOLDEN, "selftest21.llmq"), str(out)], capture_output=True, text=True,
                       env=env, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    d = np.load(os.path.join(GOLDEN, "selftest21.npz"))
    got = np.fromfile(out, np.float32).reshape(d["logits"].shape)
    assert np.array_equal(got.view(np.uint32), d["logits"].view(np.uint32))
    lines = r.stdout.split()
    ids = [int(v) for v in lines[:6]]
    assert ids == d["logits"].argmax(axis=1).tolist()
    assert lines[6:] == ["len", "6"]
