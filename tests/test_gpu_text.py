"""Text backbone parity through the C ABI against the CPU oracle, per precision profile
(src/verify.rs:66-110): embeddings and their 512/256/128 Matryoshka cuts."""
import json
import zlib
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from conftest import pkg

B = pkg("backend")
V = pkg("verify")
L = pkg("lib")

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden" / "golden_text.json"


def ids_for(lens, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 262144, size=n).astype(np.uint32) for n in lens]


def check_embeddings(got: dict, want: np.ndarray, profile, label):
    """Checks every vector and cut, prints the worst margins, then fails on any violation."""
    checks = []
    for i in range(want.shape[0]):
        checks.append(V.vec_check(f"{label}[{i}]", got[768][i], want[i], profile.embedding))
        for d in (512, 256, 128):
            cut = O.truncate_and_normalize(want[i:i + 1], d)[0]
            checks.append(V.vec_check(f"{label}[{i}]@{d}", got[d][i], cut, profile.embedding))
    worst = max(c.max_abs for c in checks)
    min_cos = min(c.cos for c in checks if c.cos is not None)
    print(f"{label}: n={len(checks)} worst max|d|={worst:.3e} min cos={min_cos:.8f}")
    bad = [str(c) for c in checks if not c.passed()]
    assert not bad, "\n".join(bad)
    return worst


@pytest.fixture(scope="module")
def cases(oracle_text):
    out = {}
    # "short" and "queries": short sequences share attention tiles (several groups, closed by a long
    # sequence or by the tile size).
    for name, lens in {"short": [17, 3, 27, 1], "doc": [700], "mixed": [130, 600, 64, 65, 1100],
                       "queries": [5, 64, 9, 33, 120, 1, 61, 300, 17, 17, 17, 40, 2, 90, 127, 128, 31, 33]}.items():
        seqs = ids_for(lens, zlib.crc32(name.encode()) % 1000)
        out[name] = (seqs, oracle_text.embed_ids(seqs))
    return out


@pytest.mark.parametrize("prec", ["bf16", "tf32", "f32"])
def test_embed_ids_parity(prec, cases, request):
    dev = request.getfixturevalue(f"dev_{prec}")
    tb = B.TextBackend(dev)
    prof = V.for_precision(prec)
    for name, (seqs, want) in cases.items():
        got = tb.embed_ids(seqs)
        w = check_embeddings(got, want, prof, f"{prec}/{name}")
        print(f"{prec} {name}: worst max|d| {w:.2e}")


@pytest.mark.parametrize("prec", ["bf16", "f32"])
def test_forward_packed_rows(prec, oracle_text, request):
    """The drop-in call itself: per-token states [rows, 768] for host embeddings."""
    dev = request.getfixturevalue(f"dev_{prec}")
    tb = B.TextBackend(dev)
    lens = [5, 64, 200]
    seqs = ids_for(lens, 9)
    ids = np.concatenate(seqs)
    e = oracle_text.embed_tokens(ids)
    np.testing.assert_array_equal(tb.embed_tokens(ids), e)
    got = tb.forward_packed(e, lens)
    want = oracle_text.forward_packed(e, lens)
    tol = 2e-5 if prec == "f32" else 0.08
    assert np.abs(got - want).max() < tol * max(1.0, float(np.abs(want).max()))
    if prec != "f32":
        assert V.cosine(got, want) > 0.9999


def test_golden_through_gpu(dev_bf16):
    g = json.loads(GOLDEN.read_text())
    tb = B.TextBackend(dev_bf16)
    for case in g["cases"]:
        got = tb.embed_ids([np.asarray(x, dtype=np.uint32) for x in case["ids"]])
        for i, o in enumerate(case["outputs"]):
            for key, d in (("emb", 768), ("emb512", 512), ("emb256", 256), ("emb128", 128)):
                c = V.vec_check(f"golden {case['name']}[{i}]@{d}", got[d][i], o[key], V.BF16.embedding)
                assert c.passed(), str(c)


def test_long_documents_bf16(dev_bf16, oracle_text):
    """Two 2208-token documents (the metric's length) against the oracle."""
    seqs = ids_for([2208, 2208], 21)
    want = oracle_text.embed_ids(seqs)
    got = B.TextBackend(dev_bf16).embed_ids(seqs)
    check_embeddings(got, want, V.BF16, "bf16/2208")


def test_errors_leave_output_untouched(dev_bf16):
    tb = B.TextBackend(dev_bf16)
    with pytest.raises(L.Eg2Error):
        tb.embed_ids([np.array([1, 2], np.uint32), np.array([], np.uint32)])
    with pytest.raises(L.Eg2Error):
        tb.embed_ids([np.array([1, 262144], np.uint32)])
    with pytest.raises(L.Eg2Error):
        tb.embed_ids([np.array([1, 2], np.uint32)], dims=(769,))
    out = np.full((2, 768), 7.0, np.float32)
    lib = L.load()
    rc = lib.eg2_forward_packed(dev_bf16.handle, np.zeros((2, 512), np.float32).ctypes.data, L.i32_array([2, 0]), 2,
                                out.ctypes.data)
    assert rc == -1 and np.all(out == 7.0)
    # The context stays usable after errors.
    got = tb.embed_ids([np.array([5, 6, 7], np.uint32)])
    assert np.isfinite(got[768]).all()


def test_repeated_calls_are_deterministic(dev_bf16):
    tb = B.TextBackend(dev_bf16)
    seqs = ids_for([300, 17], 4)
    a = tb.embed_ids(seqs)[768].copy()
    b = tb.embed_ids(seqs)[768].copy()
    np.testing.assert_array_equal(a, b)


def test_add_norm_fusion_matches_kernel_path(cases, request, monkeypatch):
    """The o / down / ple_proj GEMMs with the residual update and norms in their epilogue (2-CTA
    clusters exchanging row sums of squares) against the GEMM + add_norm kernel path. The fused
    epilogue runs on passes above 4,096 rows (smaller ones split K), hence the extra 2,200 tokens."""
    dev = request.getfixturevalue("dev_bf16")
    tb = B.TextBackend(dev)
    seqs = cases["mixed"][0] + cases["short"][0] + ids_for([2200], 77)
    assert sum(len(x) for x in seqs) > 4096
    fused = tb.embed_ids(seqs)
    monkeypatch.setenv("EG2_NO_ADD_NORM_FUSION", "1")
    plain = tb.embed_ids(seqs)
    for d in (768, 128):
        diff = np.abs(fused[d] - plain[d]).max()
        cos = (fused[d] * plain[d]).sum(1) / (np.linalg.norm(fused[d], axis=1) * np.linalg.norm(plain[d], axis=1))
        print(f"fused vs kernel path @{d}: max|d| {diff:.2e} min cos {cos.min():.8f}")
        assert diff <= 2e-3 and cos.min() >= 0.99995
