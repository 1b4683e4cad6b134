"""Shared fixtures.  GPU tests carry @pytest.mark.gpu and are skipped only when
the machine has no NVIDIA device at all; on a GPU box a missing or broken
library makes them fail."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "llm-project_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

GOLDEN = os.path.join(ROOT, "tests", "golden")


def reference_dir() -> str | None:
    """The reference checkout ($LLMQ_REFERENCE_DIR, else a directory named
    `reference` beside this repository) when it is present; None elsewhere
    (the GPU box has none)."""
    for d in (os.environ.get("LLMQ_REFERENCE_DIR"), os.path.join(os.path.dirname(ROOT), "reference")):
        if d and os.path.exists(os.path.join(d, "llama.h")):
            return d
    return None


def has_gpu() -> bool:
    return os.path.exists("/dev/nvidiactl") or os.path.exists("/dev/nvidia0")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="no NVIDIA GPU on this machine")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def _ensure_built():
    import llmq
    orc = os.path.join(ROOT, "oracle", "_build", "liboracle.so")
    if not os.path.exists(orc):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True, capture_output=True)
    cli = os.path.join(ROOT, "llm-project_b200", "bin", "llmq_run")
    if not os.path.exists(llmq.LIB_PATH) or not os.path.exists(cli):
        subprocess.run(["make", "-C", os.path.join(ROOT, "llm-project_b200", "csrc")], check=True,
                       capture_output=True)


@pytest.fixture(scope="session")
def lib():
    _ensure_built()
    import llmq
    return llmq.load()


@pytest.fixture(scope="session")
def orc():
    _ensure_built()
    import oracle
    return oracle.load_oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle
    r = oracle.load_reference()
    if r is None:
        pytest.skip("reference build (oracle/_ref) not available")
    return r
