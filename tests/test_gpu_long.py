"""The reference's long case (C4): one sequence of 11,774 tokens (README.md:46), through the C ABI,
against the CPU oracle's result for the same ids (computed once by tests/golden/make_oracle_fixtures.py
-- the oracle needs minutes at this length -- and committed). Every precision meets its own profile
(src/verify.rs:66-110).
"""
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import pkg
from test_gpu_text import check_embeddings

sys.path.insert(0, str(Path(__file__).parent / "golden"))
import make_oracle_fixtures as M  # noqa: E402

B = pkg("backend")
V = pkg("verify")

pytestmark = pytest.mark.gpu
FIXTURES = Path(__file__).parent / "golden" / "oracle_fixtures.npz"


@pytest.mark.parametrize("prec", ["bf16", "tf32", "f32"])
def test_long_sequence_against_oracle(prec, request):
    f = np.load(FIXTURES)
    seqs = M.case_ids("c4")
    assert [len(x) for x in seqs] == list(f["c4_lens"]) == [11774]
    got = B.TextBackend(request.getfixturevalue(f"dev_{prec}")).embed_ids(seqs)
    check_embeddings(got, f["c4_emb"], V.for_precision(prec), f"{prec}/long11774")
