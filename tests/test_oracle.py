"""The CPU oracle, pinned before it is trusted.

* against golden vectors made from transformers' Gemma4 modules on the same seeded checkpoint
  (tests/golden/make_golden.py for the text backbone, make_golden_vision.py for the vision tower) -- the
  upstream implementation the reference's own dumps come from;
* op by op against exact float64 restatements (the method of examples/check_attention.rs:31-52);
* packing: a packed pass equals its sequences run one by one (src/text.rs:131-135).
"""
import base64
import json
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from conftest import pkg

V = pkg("verify")
GOLDEN = Path(__file__).parent / "golden" / "golden_text.json"
GOLDEN_VISION = Path(__file__).parent / "golden" / "golden_vision.json"


def exact_attention(q, k, v, lens, nh, nkv, hd, window):
    """float64 block-diagonal attention (examples/check_attention.rs:31-52)."""
    out = np.zeros((q.shape[0], nh * hd))
    off = 0
    for L in lens:
        for h in range(nh):
            g = h // (nh // nkv)
            qh = q[off:off + L, h * hd:(h + 1) * hd].astype(np.float64)
            kh = k[off:off + L, g * hd:(g + 1) * hd].astype(np.float64)
            vh = v[off:off + L, g * hd:(g + 1) * hd].astype(np.float64)
            s = qh @ kh.T
            if window is not None:
                i = np.arange(L)
                s = np.where(np.abs(i[:, None] - i[None, :]) <= window, s, -np.inf)
            s = s - s.max(1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(1, keepdims=True)
            out[off:off + L, h * hd:(h + 1) * hd] = p @ vh
        off += L
    return out


@pytest.fixture(scope="module")
def golden():
    return json.loads(GOLDEN.read_text())


def test_oracle_matches_golden(oracle_text, golden):
    for case in golden["cases"]:
        emb = oracle_text.embed_ids(case["ids"])
        for i, want in enumerate(case["outputs"]):
            c = V.vec_check(f"{case['name']}[{i}]", emb[i], want["emb"], V.FLOAT32.embedding)
            assert c.passed(), str(c)
            for d in (512, 256, 128):
                cut = O.truncate_and_normalize(emb[i:i + 1], d)[0]
                c = V.vec_check(f"{case['name']}[{i}]@{d}", cut, want[f"emb{d}"], V.FLOAT32.embedding)
                assert c.passed(), str(c)


def test_oracle_rows_match_golden(oracle_text, golden):
    # Per-token states before pooling: first and last row of each sequence.
    for case in golden["cases"]:
        ids = np.concatenate([np.asarray(x, dtype=np.uint32) for x in case["ids"]])
        hs = oracle_text.forward_packed(oracle_text.embed_tokens(ids), case["lens"])
        off = 0
        for L, rows in zip(case["lens"], case["rows"]):
            assert np.abs(hs[off] - np.asarray(rows["first"])).max() < 2e-5
            assert np.abs(hs[off + L - 1] - np.asarray(rows["last"])).max() < 2e-5
            off += L


def test_packed_equals_separate(oracle_text):
    rng = np.random.default_rng(3)
    lens = [5, 130, 1]
    ids = rng.integers(0, 262144, size=sum(lens)).astype(np.uint32)
    e = oracle_text.embed_tokens(ids)
    packed = oracle_text.forward_packed(e, lens)
    off = 0
    for L in lens:
        single = oracle_text.forward_packed(e[off:off + L], [L])
        np.testing.assert_array_equal(single, packed[off:off + L])
        off += L


@pytest.mark.parametrize("nh,nkv,hd,window", [(4, 2, 256, 512), (4, 2, 256, 7), (4, 1, 512, None), (12, 12, 64, None)])
def test_attention_oracle_vs_exact(nh, nkv, hd, window):
    rng = np.random.default_rng(7)
    lens = [1, 33, 129, 300]
    rows = sum(lens)
    sigma = hd ** -0.25
    q = (rng.standard_normal((rows, nh * hd)) * sigma).astype(np.float32)
    k = (rng.standard_normal((rows, nkv * hd)) * sigma).astype(np.float32)
    v = rng.standard_normal((rows, nkv * hd)).astype(np.float32)
    got = O.attention_packed(q, k, v, lens, nh, nkv, hd, window)
    want = exact_attention(q, k, v, lens, nh, nkv, hd, window)
    assert np.abs(got - want).max() < 2e-5


def test_sgemm_vs_numpy():
    rng = np.random.default_rng(1)
    for m, n, k in [(17, 2048, 512), (3, 768, 512), (130, 512, 2048), (1, 256, 8), (5, 7, 3)]:
        x = rng.standard_normal((m, k)).astype(np.float32)
        w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)
        got = O.sgemm_nt(x, w)
        want = x.astype(np.float64) @ w.astype(np.float64).T
        assert np.abs(got - want).max() < 1e-4


def test_gelu_constants():
    for x in (-3.0, -0.5, 0.0, 0.7, 2.5):
        ref = 0.5 * x * (1 + np.tanh(np.float32(0.79788456) * (x + 0.044715 * x ** 3)))
        assert abs(O.gelu_tanh(x) - ref) < 1e-6


def test_pool_and_matryoshka():
    rng = np.random.default_rng(2)
    h = rng.standard_normal((10, 768)).astype(np.float32)
    p = O.pool(h, [3, 7])
    for s, (a, b) in enumerate([(0, 3), (3, 10)]):
        m = h[a:b].astype(np.float64).mean(0)
        np.testing.assert_allclose(p[s], m / np.linalg.norm(m), atol=1e-7)
    cut = O.truncate_and_normalize(p, 128)
    np.testing.assert_allclose(np.linalg.norm(cut, axis=1), 1.0, atol=1e-6)
    np.testing.assert_array_equal(O.truncate_and_normalize(p, 768), p)
    with pytest.raises(ValueError):
        O.truncate_and_normalize(p, 0)
    with pytest.raises(ValueError):
        O.truncate_and_normalize(p, 769)


def test_empty_sequence_rejected(oracle_text):
    with pytest.raises(ValueError):
        oracle_text.forward_packed(np.zeros((3, 512), np.float32), [3, 0])


def test_vision_oracle_shapes(oracle_vision):
    rng = np.random.default_rng(4)
    gh, gw = 6, 9
    patches = rng.random((gh * gw, 768), dtype=np.float32)
    pos = np.array([[x, y] for y in range(gh) for x in range(gw)], dtype=np.int32)
    pooled, soft = oracle_vision.encode(patches, pos, gh, gw)
    assert pooled.shape == (6, 768) and soft.shape == (6, 512)
    assert np.isfinite(soft).all()
    with pytest.raises(ValueError):
        oracle_vision.encode(patches[:50], pos[:50], 5, 10)


def test_vision_oracle_matches_golden(oracle_vision):
    """The vision tower (src/vision.rs:223-273) and the multimodal embedder against transformers'
    Gemma4VisionModel + Gemma4MultimodalEmbedder on the same checkpoint and patches: 6 x 6, 3 x 9 and
    3 x 3 grids (4, 3 and 1 soft tokens). The pooled states carry the sqrt(768) scale (hundreds), so
    they are compared relative to their largest magnitude; the soft tokens are O(1)."""
    g = json.loads(GOLDEN_VISION.read_text())
    for case in g["cases"]:
        gh, gw = case["grid"]
        patches = np.frombuffer(base64.b64decode(case["patches_f32_b64"]), dtype="<f4").reshape(gh * gw, -1)
        pos = np.array(case["positions"], dtype=np.int32)
        pooled, soft = oracle_vision.encode(patches, pos, gh, gw)
        pw, sw = np.array(case["pooled"], np.float32), np.array(case["soft"], np.float32)
        assert pooled.shape == pw.shape and soft.shape == sw.shape
        assert np.abs(pooled - pw).max() <= 1e-5 * np.abs(pw).max(), (gh, gw)
        assert np.abs(soft - sw).max() <= 1e-5, (gh, gw)


def test_oracle_fixtures_match_this_checkpoint_and_c1(oracle_text, tmp_path):
    """The committed oracle fixtures (tests/golden/oracle_fixtures.npz, written by
    make_oracle_fixtures.py) belong to this checkpoint, and the oracle reproduces their C1 case --
    BASELINE configs[0] as stated: one 512-token sequence of seed-0 uniform ids through the CPU f32
    path, pooled, L2-normalised, with its 512/256/128 cuts."""
    import sys

    golden = Path(__file__).parent / "golden"
    sys.path.insert(0, str(golden))
    import make_oracle_fixtures as M

    f = np.load(golden / "oracle_fixtures.npz")
    pkg("weights").make_random_checkpoint(tmp_path, seed=0, vision=False)
    assert str(f["checkpoint_sha256"]) == M.checkpoint_sha256(tmp_path)
    seqs = M.case_ids("c1")
    got = oracle_text.embed_ids(seqs)
    np.testing.assert_allclose(got, f["c1_emb"], rtol=0, atol=1e-6)
    for d in (512, 256, 128):
        cut = O.truncate_and_normalize(got, d)
        assert cut.shape == (1, d) and abs(np.linalg.norm(cut) - 1) < 1e-6
    assert [len(x) for x in M.case_ids("c3")] == list(f["c3_lens"])
    assert [len(x) for x in M.case_ids("c4")] == list(f["c4_lens"])
