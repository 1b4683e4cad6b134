"""GPU failure detection without a fault: every device-side wait on another
rank's flag is bounded.  A two-rank exchange whose second rank never raises its
flag is run on one GPU with a short poll limit; the kernel must return by
itself with the timeout bit in the error word, the host call must report the
error, and the device must stay usable (a decode step afterwards is still
bit-identical to the oracle)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from helpers import TINY, bits_equal, gpu_decode, orc_decode, synth

pytestmark = pytest.mark.gpu

ERR_TIMEOUT = 1
LLMQ_ERR_CUDA = 2


@pytest.mark.parametrize("which", [0, 1], ids=["absmax_exchange", "row_parallel_gemv"])
def test_peer_flag_wait_gives_up_and_reports(lib, orc, which):
    err, ms = C.c_int(0), C.c_float(0.0)
    rc = lib.llmq_tp_wait_timeout_check(which, 4096, C.byref(err), C.byref(ms))
    assert rc == LLMQ_ERR_CUDA, lib.q_llama_last_error_message()
    assert err.value & ERR_TIMEOUT
    assert b"error flags" in lib.q_llama_last_error_message()
    assert 0.0 < ms.value < 500.0  # a few thousand ~32 ns polls, not the production second
    lib.q_llama_clear_error()
    # the context is intact: the next decode is still the oracle's, bit for bit
    m = synth(lib, TINY, seed=11)
    ids = [3, 1, 4, 1, 5]
    got, _ = gpu_decode(lib, m, ids)
    want, _ = orc_decode(orc, m, ids)
    assert bits_equal(got, want)
    lib.q_llama_model_free(C.byref(m))
