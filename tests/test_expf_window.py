"""CPU: the device expf's fast paths (libm_expf in llmq_kernels.cuh) decide
from the 29 mantissa bits that the double-to-float rounding of y = exp((double)x)
drops, instead of bracketing y between its float neighbours.  For the same y,
those decisions must be lx_expf_cr's (libm_expf.h): far from the rounding
midpoint the result is (float)y; near it but decidable by y, the correctly
rounded float and the neighbour on the other side of y.  tests/expf_window_check.c
restates them and compares on every 13th binary32 input.  (The device routine
as a whole is compared with the host libm on all 2^32 inputs on the GPU.)"""
from __future__ import annotations

import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_expf_fast_path_decisions_equal_the_bracket(tmp_path):
    src = os.path.join(ROOT, "tests", "expf_window_check.c")
    exe = str(tmp_path / "expf_window_check")
    subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-I", os.path.join(ROOT, "llm-project_b200", "csrc"),
                    "-o", exe, src, "-lm"], check=True)
    r = subprocess.run([exe, "13"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert " 0 mismatches" in r.stdout
