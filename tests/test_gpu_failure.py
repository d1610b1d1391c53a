"""Failure detection on the GPU without a fault: a device-side wait that nothing satisfies runs out
after its wall-time limit, records its status, and the context stays usable (every pipeline barrier
of the library waits this way; the host reports a recorded status as EG2_ERR_TIMEOUT)."""
import ctypes as C
import time

import numpy as np
import pytest

from conftest import pkg

L = pkg("lib")

pytestmark = pytest.mark.gpu
EG2_DEV_TIMEOUT_PROBE = 4


def test_bounded_wait_runs_out_and_context_survives():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = L.load()
    st = C.c_int(-1)
    t0 = time.perf_counter()
    rc = lib.eg2_wait_timeout_probe(0, 20000, C.byref(st))  # 20 ms limit
    dt = time.perf_counter() - t0
    assert rc == 0
    assert st.value == EG2_DEV_TIMEOUT_PROBE
    assert dt >= 0.02
    assert lib.eg2_device_status() == 0  # cleared by the probe call
    # The context still runs work: a small bf16 GEMM through the C ABI.
    M, N, K = 128, 256, 64
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    c = torch.empty(M, N, device="cuda", dtype=torch.float32)
    rc = lib.eg2_gemm(2, a.data_ptr(), K, w.data_ptr(), K, c.data_ptr(), N, M, N, K, 1, None)
    torch.cuda.synchronize()
    assert rc == 0
    ref = a.float() @ w.float().t()
    assert torch.allclose(c, ref, rtol=1e-2, atol=1e-2)


def test_probe_rejects_bad_arguments():
    lib = L.load()
    st = C.c_int(0)
    assert lib.eg2_wait_timeout_probe(0, 0, C.byref(st)) != 0
    assert lib.eg2_wait_timeout_probe(0, 3000000, C.byref(st)) != 0
