"""GPU: qmatmul_device_noalloc, the entry point for callers that cannot allocate
device memory where they multiply (for example a framework whose memory pool
owns the GPU).  It must give exactly what the allocating qmatmul gives, call
after call, since every call reuses the same fixed scratch array inside the
library.  Collected last on purpose (file name) so a failure here does not stop
the other GPU tests; it also passes alone in a fresh process."""
from __future__ import annotations

import numpy as np
import pytest

import llmq
from helpers import bits_equal, gpu_qmatmul

pytestmark = pytest.mark.gpu


def _device(arr):
    import torch
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


@pytest.mark.parametrize("M,K,N", [(1, 4096, 4096), (3, 37, 19), (2, 14336, 1000), (1, 288, 131072)])
def test_noalloc_matches_qmatmul_twice(lib, M, K, N):
    import torch
    rng = np.random.default_rng(M * 100003 + K * 17 + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    A[0, : min(K, 4)] = [127.0, 0.5, 1.5, -2.5][: min(K, 4)]
    q = rng.integers(-127, 128, size=(K, N)).astype(np.int8)
    s = rng.uniform(1e-3, 1e-2, size=N).astype(np.float32)
    expect = gpu_qmatmul(lib, A, q, s)  # the existing, allocating entry point
    dA, dq, ds = _device(A), _device(q), _device(s)
    for call in range(2):  # twice: the shared scratch must be left clean
        dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        rc = lib.qmatmul_device_noalloc(dA.data_ptr(), M, K, dq.data_ptr(), ds.data_ptr(), N, dC.data_ptr(), None)
        assert rc == 0, lib.q_llama_last_error_message()
        torch.cuda.synchronize()
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
