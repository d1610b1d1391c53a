"""eg2_attention_noalloc through the C ABI, against eg2_attention (kind EG2_BF16) on the same inputs.

The allocation-free entry point is for callers that cannot call cudaMalloc: engines that hand all
device memory to their own pool up front, and latency-critical paths that cannot take cudaMalloc's
implicit device synchronisation. Its scratch (sequence lengths and the query-tile list) sits in one
fixed device array that every call shares and that keeps the last call's contents, so the test makes
calls in a row with different shapes: each must match the allocating entry point exactly (both run
the same tensor-core kernel over the same tile list), and a later call must not pick up anything a
previous one left behind. The call reports a bounded device wait that ran out only through the
device status word, which the test reads after synchronising.

This file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import pkg

L = pkg("lib")
W = pkg("weights")
torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _inputs(rows, nh, nkv, hd, seed):
    rng = np.random.default_rng(seed)
    sigma = hd ** -0.25
    q = W.f32_to_bf16_bits((rng.standard_normal((rows, nh * hd)) * sigma).astype(np.float32))
    k = W.f32_to_bf16_bits((rng.standard_normal((rows, nkv * hd)) * sigma).astype(np.float32))
    v = W.f32_to_bf16_bits(rng.standard_normal((rows, nkv * hd)).astype(np.float32))
    return [torch.from_numpy(a.view(np.int16)).cuda() for a in (q, k, v)]


def _run(fn, q, k, v, lens, nh, nkv, hd, window):
    out = torch.full((q.shape[0], nh * hd), 0x40E0, dtype=torch.int16, device="cuda")
    rc = fn(C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), C.c_void_p(out.data_ptr()),
            L.i32_array(lens), len(lens), nh, nkv, hd, window, None)
    torch.cuda.synchronize()
    assert rc == 0, L.ERRORS.get(rc, rc)
    return out.cpu().numpy()


def _allocating(*args):
    return L.load().eg2_attention(L.EG2_BF16, *args)


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls():
    lib = L.load()
    cases = [
        # sliding-window layer shape, many short and some long sequences
        ([5, 64, 65, 300, 1, 700] + [17] * 40, 4, 2, 256, 512),
        # global layer shape with fewer, longer sequences (different tile size and count)
        ([2208, 33, 900], 4, 1, 512, -1),
        # a short call after the long ones: only its own tiles may be used
        ([3, 70], 4, 2, 256, 512),
    ]
    for i, (lens, nh, nkv, hd, window) in enumerate(cases):
        q, k, v = _inputs(sum(lens), nh, nkv, hd, seed=100 + i)
        got = _run(lib.eg2_attention_noalloc, q, k, v, lens, nh, nkv, hd, window)
        want = _run(_allocating, q, k, v, lens, nh, nkv, hd, window)
        assert lib.eg2_device_status() == 0
        assert np.isfinite(W.bf16_bits_to_f32(got.view(np.uint16))).all()
        np.testing.assert_array_equal(got, want)


def test_noalloc_rejects_calls_beyond_its_fixed_scratch():
    """Every rejection happens on the host before anything is copied or launched. The q / k / v / out
    buffers are nonetheless sized for the rows each call describes, so that a call the limits failed to
    catch would still stay inside its buffers."""
    lib = L.load()

    def call(lens, nh=4, nkv=2, hd=256, window=512):
        rows = max(1, sum(max(0, x) for x in lens))
        q = torch.zeros((rows, max(1, nh) * hd), dtype=torch.int16, device="cuda")
        kv = torch.zeros((rows, max(1, nkv) * hd), dtype=torch.int16, device="cuda")
        out = torch.full((rows, max(1, nh) * hd), 7, dtype=torch.int16, device="cuda")
        rc = lib.eg2_attention_noalloc(C.c_void_p(q.data_ptr()), C.c_void_p(kv.data_ptr()), C.c_void_p(kv.data_ptr()),
                                       C.c_void_p(out.data_ptr()), L.i32_array(lens), len(lens), nh, nkv, hd, window,
                                       None)
        torch.cuda.synchronize()
        assert bool((out == 7).all()), "a rejected call wrote its output"
        return rc

    # Query tokens per tile: 128 for 4 query heads over 2 K/V heads of 256, 64 for 4 over 1 of 512.
    assert call([1] * 65537) == -1                      # more sequences than the array holds
    assert call([129] + [1] * 65535) == -1              # 65,536 sequences, but 65,537 query tiles
    assert call([65] + [1] * 65535, nkv=1, hd=512, window=-1) == -1  # the same with 64-token tiles
    assert call([5, 0, 3]) == -1                        # an empty sequence
    assert call([5, -2]) == -1                          # a negative length
    assert call([8], nh=0) == -1                        # no query heads
    assert call([8], nkv=0) == -1                       # no K/V heads
    assert call([8], nh=4, nkv=3) == -1                 # query heads not a multiple of K/V heads
    assert call([8], hd=128) == -1                      # a head size the kernels do not take
    assert lib.eg2_device_status() == 0
