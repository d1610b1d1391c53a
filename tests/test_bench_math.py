"""The algorithmic work bench.py divides by when it reports TFLOP/s and roofline fractions: GEMM FLOPs
per token and attention FLOPs per document, recomputed here by hand from the layer shapes and by
brute-force counting of the (query, key) pairs that the sliding window keeps."""
import tempfile
from pathlib import Path
from types import SimpleNamespace

import numpy as np

import bench
from conftest import pkg

C = pkg("config")
W = pkg("weights")


def model_config():
    d = Path(tempfile.mkdtemp())
    W.write_config(d, C.synthetic_config())
    return C.ModelConfig.load(d)


def test_gemm_flops_per_token_by_hand():
    # Sliding layer: QKV 2048 x 512, O 512 x 1024, gate|up 4096 x 512, down 512 x 2048, PLE gate and
    # projection 512 x 512 each. Global layer: QKV 3072 x 512, O 512 x 2048, the rest the same.
    sliding = 2 * (2048 * 512 + 512 * 1024 + 4096 * 512 + 512 * 2048 + 2 * 512 * 512)
    global_ = 2 * (3072 * 512 + 512 * 2048 + 4096 * 512 + 512 * 2048 + 2 * 512 * 512)
    once = 2 * (24 * 512 * 512) + 2 * (768 * 512)  # PLE model projection, 512 -> 768 output
    want = 20 * sliding + 4 * global_ + once
    assert want == 273_416_192
    assert bench.gemm_flops_per_token(model_config()) == want


def _fake_cfg(layers, window, heads, sliding_hd=256, global_hd=512, every=6):
    def is_sliding(i):
        return i % every != every - 1

    def layer_dims(i):
        return (sliding_hd, 2) if is_sliding(i) else (global_hd, 1)

    text = SimpleNamespace(sliding_window=window, num_hidden_layers=layers, num_attention_heads=heads,
                           is_sliding=is_sliding, layer_dims=layer_dims)
    return SimpleNamespace(text=text)


def test_attention_flops_counts_the_window_pairs():
    for L, window in ((1, 3), (7, 3), (40, 5), (64, 64), (100, 512)):
        cfg = _fake_cfg(layers=6, window=window, heads=4)
        i = np.arange(L)
        pairs_sliding = int((np.abs(i[:, None] - i[None, :]) <= window).sum())
        want = 5 * 4 * 4 * 256 * pairs_sliding + 1 * 4 * 4 * 512 * L * L
        assert bench.attention_flops(cfg, L) == want, (L, window)


def test_attention_flops_of_the_benchmark_document():
    # 2,208 tokens, 20 sliding layers (radius 512) and 4 global ones: 323.6 GFLOP per document.
    f = bench.attention_flops(model_config(), 2208)
    assert abs(f / 1e9 - 323.637) < 1e-3
