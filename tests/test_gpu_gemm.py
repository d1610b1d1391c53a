"""GEMM sweep through the C ABI against the CPU oracle's f32 GEMM.

Shapes: every projection of a text layer (QKV sliding/global, O, gate|up, down, PLE gate/proj),
the PLE model projection and the 512 -> 768 output projection, at M = 17, 512, 2208 (8192 for a
subset). X ~ N(0, 1), W ~ N(0, 1/K). The reference for bf16 is the f32 GEMM of the bf16-rounded
inputs, so only accumulation order separates the two.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from conftest import pkg

L = pkg("lib")
W = pkg("weights")
torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

SHAPES = [(2048, 512), (3072, 512), (512, 1024), (512, 2048), (4096, 512), (512, 512), (12288, 512), (768, 512)]


def run_gemm(kind, x, w, out_f32=True):
    lib = L.load()
    m, k = x.shape
    n = w.shape[0]
    if kind == L.EG2_BF16:
        xd = torch.from_numpy(W.f32_to_bf16_bits(x).view(np.int16)).cuda()
        wd = torch.from_numpy(W.f32_to_bf16_bits(w).view(np.int16)).cuda()
    else:
        xd = torch.from_numpy(x).cuda()
        wd = torch.from_numpy(w).cuda()
    dt = torch.float32 if (out_f32 or kind != L.EG2_BF16) else torch.int16
    # Sentinel rows past M must stay untouched.
    out = torch.full((m + 3, n), 7.0 if dt == torch.float32 else 0x40E0, dtype=dt, device="cuda")
    rc = lib.eg2_gemm(kind, C.c_void_p(xd.data_ptr()), k, C.c_void_p(wd.data_ptr()), k, C.c_void_p(out.data_ptr()), n,
                      m, n, k, 1 if out_f32 else 0, None)
    torch.cuda.synchronize()
    assert rc == 0, L.ERRORS.get(rc, rc)
    assert lib.eg2_device_status() == 0
    o = out.cpu().numpy()
    if dt == torch.int16:
        o = W.bf16_bits_to_f32(o.view(np.uint16))
        assert np.all(o[m:] == 7.0)
    else:
        assert np.all(o[m:] == 7.0)
    return o[:m]


def data(m, n, k, seed=0):
    rng = np.random.default_rng(seed + m * 7 + n * 3 + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)
    return x, w


@pytest.mark.parametrize("m", [17, 512, 2208])
@pytest.mark.parametrize("n,k", SHAPES)
def test_bf16_gemm_sweep(m, n, k):
    x, w = data(m, n, k)
    xr, wr = W.bf16_round(x), W.bf16_round(w)
    want = O.sgemm_nt(xr, wr)
    got = run_gemm(L.EG2_BF16, x, w)
    assert np.abs(got - want).max() < 2e-4 * max(1.0, float(np.abs(want).max()))


@pytest.mark.parametrize("n,k", [(4096, 512), (512, 2048)])
def test_bf16_gemm_large_m(n, k):
    x, w = data(8192, n, k)
    want = O.sgemm_nt(W.bf16_round(x), W.bf16_round(w))
    got = run_gemm(L.EG2_BF16, x, w)
    assert np.abs(got - want).max() < 2e-4 * max(1.0, float(np.abs(want).max()))


@pytest.mark.parametrize("m", [1, 128, 129, 255, 256, 257, 383, 1000])
def test_bf16_gemm_pair_tile_edges(m):
    """bf16 GEMMs run on CTA pairs (256-row tiles, 128 rows per CTA): row counts that leave the
    odd CTA of the last pair empty, partly filled or full."""
    x, w = data(m, 2048, 512, seed=3)
    want = O.sgemm_nt(W.bf16_round(x), W.bf16_round(w))
    got = run_gemm(L.EG2_BF16, x, w)
    assert np.abs(got - want).max() < 2e-4 * max(1.0, float(np.abs(want).max()))
    got_b = run_gemm(L.EG2_BF16, x, w, out_f32=False)
    np.testing.assert_array_equal(W.bf16_round(got), got_b)


def test_bf16_output_is_rounded_f32_accumulator():
    x, w = data(300, 1024, 512)
    f = run_gemm(L.EG2_BF16, x, w, out_f32=True)
    b = run_gemm(L.EG2_BF16, x, w, out_f32=False)
    np.testing.assert_array_equal(W.bf16_round(f), b)


@pytest.mark.parametrize("m", [17, 2208])
@pytest.mark.parametrize("n,k", [(2048, 512), (512, 2048), (768, 512)])
def test_tf32_gemm(m, n, k):
    x, w = data(m, n, k, seed=1)
    want = x.astype(np.float64) @ w.astype(np.float64).T
    got = run_gemm(L.EG2_TF32, x, w)
    err = np.abs(got - want)
    assert err.max() < 1e-2 and err.mean() < 1e-3


@pytest.mark.parametrize("m,n,k", [(17, 2048, 512), (513, 768, 512), (200, 512, 2048)])
def test_f32_gemm(m, n, k):
    x, w = data(m, n, k, seed=2)
    want = O.sgemm_nt(x, w)
    got = run_gemm(L.EG2_F32, x, w)
    assert np.abs(got - want).max() < 2e-5


def test_gemm_rejects_unsupported_shapes():
    lib = L.load()
    x = torch.zeros((4, 100), dtype=torch.int16, device="cuda")
    w = torch.zeros((256, 100), dtype=torch.int16, device="cuda")
    o = torch.zeros((4, 256), dtype=torch.float32, device="cuda")
    rc = lib.eg2_gemm(L.EG2_BF16, C.c_void_p(x.data_ptr()), 100, C.c_void_p(w.data_ptr()), 100, C.c_void_p(o.data_ptr()),
                      256, 4, 256, 100, 1, None)
    assert rc == -1
