"""The reference's long case (C4): one sequence of 11,774 tokens (README.md:46), through the C ABI.

The CPU oracle needs minutes at this length, so the f32 path of the library stands in for it: at
every shorter length the tests check it against the oracle to ~1e-6 (float32 profile 5e-6), and
here the bf16 and TF32 paths must meet their own profiles (src/verify.rs:66-110) against it.
"""
import numpy as np
import pytest

from conftest import pkg
from test_gpu_text import check_embeddings

B = pkg("backend")
V = pkg("verify")

pytestmark = pytest.mark.gpu
LONG = 11774


@pytest.fixture(scope="module")
def long_ids():
    rng = np.random.default_rng(11774)
    return [rng.integers(0, 262144, size=LONG).astype(np.uint32)]


@pytest.fixture(scope="module")
def f32_embedding(long_ids, request):
    dev = request.getfixturevalue("dev_f32")
    got = B.TextBackend(dev).embed_ids(long_ids)
    return np.stack([got[768][0]])


@pytest.mark.parametrize("prec", ["bf16", "tf32"])
def test_long_sequence_against_f32(prec, long_ids, f32_embedding, request):
    dev = request.getfixturevalue(f"dev_{prec}")
    got = B.TextBackend(dev).embed_ids(long_ids)
    check_embeddings(got, f32_embedding, V.for_precision(prec), f"{prec}/long{LONG}")
