"""GPU: qmatmul_device_noalloc, the entry point for callers that cannot allocate
device memory where they multiply (for example a framework whose memory pool
owns the GPU, or a plugin that must not change the application's device-memory
accounting).  It must give exactly what the reference's qmatmul gives, call after
call, since every call reuses the same fixed scratch array inside the library.
The checker is the oracle (the reference's arithmetic restated on the CPU); the
allocating GPU entry point is compared as well.  Collected last on purpose (file
name) so a failure here does not stop the other GPU tests; it also passes alone
in a fresh process."""
from __future__ import annotations

import numpy as np
import pytest

from helpers import bits_equal, gpu_qmatmul, orc_qmatmul

pytestmark = pytest.mark.gpu


def _device(arr):
    import torch
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def _inputs(M, K, N, zero_row=None):
    rng = np.random.default_rng(M * 100003 + K * 17 + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    if M and K:
        A[0, : min(K, 4)] = [127.0, 0.5, 1.5, -2.5][: min(K, 4)]
    if zero_row is not None:
        A[zero_row] = 0.0  # scale falls back to 1 (quant.c:71)
    q = rng.integers(-127, 128, size=(K, N)).astype(np.int8)
    s = rng.uniform(1e-3, 1e-2, size=N).astype(np.float32)
    return A, q, s


def _noalloc(lib, dA, M, K, dq, ds, N, stream=None):
    import torch
    dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    h = None if stream is None else stream.cuda_stream
    rc = lib.qmatmul_device_noalloc(dA.data_ptr() if dA is not None else None, M, K,
                                    dq.data_ptr() if dq is not None else None, ds.data_ptr(), N, dC.data_ptr(), h)
    assert rc == 0, lib.q_llama_last_error_message()
    return dC


@pytest.mark.parametrize("M,K,N", [(1, 4096, 4096), (3, 37, 19), (2, 14336, 1000), (1, 288, 131072)])
def test_noalloc_matches_oracle_twice(lib, orc, M, K, N):
    import torch
    A, q, s = _inputs(M, K, N)
    expect = orc_qmatmul(orc, A, q, s)
    assert bits_equal(gpu_qmatmul(lib, A, q, s), expect)  # the existing, allocating entry point
    dA, dq, ds = _device(A), _device(q), _device(s)
    for call in range(2):  # twice: the shared scratch must be left clean
        dC = _noalloc(lib, dA, M, K, dq, ds, N)
        torch.cuda.synchronize()
        assert bits_equal(dC.cpu().numpy(), expect), f"call {call}"


def test_noalloc_all_zero_row_and_side_stream(lib, orc):
    import torch
    M, K, N = 3, 1000, 777
    A, q, s = _inputs(M, K, N, zero_row=1)
    expect = orc_qmatmul(orc, A, q, s)
    dA, dq, ds = _device(A), _device(q), _device(s)
    side = torch.cuda.Stream()
    torch.cuda.synchronize()
    for call in range(2):
        with torch.cuda.stream(side):
            dC = _noalloc(lib, dA, M, K, dq, ds, N, stream=side)
        side.synchronize()
        assert bits_equal(dC.cpu().numpy(), expect), f"call {call}"
    assert np.all(expect[1] == 0.0)


def test_noalloc_empty_shapes(lib, orc):
    import torch
    # M = 0: nothing to do
    ds = _device(np.ones(8, np.float32))
    dC = torch.zeros((1, 8), dtype=torch.float32, device="cuda")
    assert lib.qmatmul_device_noalloc(None, 0, 8, None, ds.data_ptr(), 8, dC.data_ptr(), None) == 0
    # K = 0: every output is as * ws * 0 = 0 (quant.c:82), with A and Wq NULL
    s = np.random.default_rng(3).uniform(1e-3, 1e-2, size=16).astype(np.float32)
    ds = _device(s)
    for call in range(2):
        dC = _noalloc(lib, None, 1, 0, None, ds, 16)
        torch.cuda.synchronize()
        expect = orc_qmatmul(orc, np.zeros((1, 0), np.float32), np.zeros((0, 16), np.int8), s)
        assert bits_equal(dC.cpu().numpy(), expect), f"call {call}"


def test_noalloc_rejects_n_beyond_its_scratch(lib):
    import torch
    N = 131072 + 1
    dA = torch.zeros((1, 8), dtype=torch.float32, device="cuda")
    dq = torch.zeros((8, 16), dtype=torch.int8, device="cuda")
    rc = lib.qmatmul_device_noalloc(dA.data_ptr(), 1, 8, dq.data_ptr(), dA.data_ptr(), N, dA.data_ptr(), None)
    assert rc == 1  # LLMQ_ERR_ARG, nothing launched
    assert b"131072" in lib.q_llama_last_error_message()
    lib.q_llama_clear_error()
