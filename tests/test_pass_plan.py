"""The pass policy of eg2_forward_packed / eg2_embed_packed (eg2_plan_passes), on the CPU.

Consecutive sequences in call order share a pass of at most ``max_rows`` rows, a longer sequence
getting a pass of its own -- the reference's greedy pack of embed_prepared (src/model.rs:508-521,
PACK_TOKENS = 2048 at :157-158), restated below as the check -- and, in bf16 contexts, sequences of at
most ``precise_max`` tokens form passes of their own that run in TF32.
"""
import numpy as np
import pytest

from conftest import pkg

B = pkg("backend")
L = pkg("lib")


def reference_pack(lens, pack_tokens):
    """embed_prepared's loop (src/model.rs:513-521): start a pack at `start`, extend it while the next
    input fits in pack_tokens rows."""
    packs, start = [], 0
    while start < len(lens):
        end, rows = start + 1, lens[start]
        while end < len(lens) and rows + lens[end] <= pack_tokens:
            rows += lens[end]
            end += 1
        packs.append(list(range(start, end)))
        start = end
    return packs


@pytest.mark.parametrize("seed", range(6))
def test_plan_matches_the_reference_greedy_pack(seed):
    rng = np.random.default_rng(seed)
    lens = [int(x) for x in rng.integers(1, 3000, size=int(rng.integers(1, 60)))]
    got = B.plan_passes(lens, 2048, 0)
    assert [p for p, _ in got] == reference_pack(lens, 2048)
    assert not any(tf32 for _, tf32 in got)


def test_short_sequences_form_their_own_passes():
    lens = [3, 2208, 5, 17, 1, 700, 16, 4000]
    got = B.plan_passes(lens, 147456, 16)
    assert got == [([1, 3, 5, 7], False), ([0, 2, 4, 6], True)]
    # Within each class the packing is the greedy one, in call order.
    got = B.plan_passes(lens, 3000, 16)
    assert got == [([1, 3, 5], False), ([7], False), ([0, 2, 4, 6], True)]


@pytest.mark.parametrize("seed", range(4))
def test_every_sequence_once_and_passes_bounded(seed):
    rng = np.random.default_rng(100 + seed)
    lens = [int(x) for x in rng.integers(1, 2500, size=400)]
    cap, pmax = 5000, 24
    plan = B.plan_passes(lens, cap, pmax)
    seen = sorted(s for p, _ in plan for s in p)
    assert seen == list(range(len(lens)))
    for seqs, tf32 in plan:
        assert seqs == sorted(seqs)
        assert all((lens[s] <= pmax) == tf32 for s in seqs)
        rows = sum(lens[s] for s in seqs)
        assert rows <= cap or len(seqs) == 1


def test_one_million_tokens_split_into_bounded_passes():
    lens = [2208] * 453 + [1000] * 3  # 1,003,224 rows; 66 documents of 2,208 fit in a pass
    plan = B.plan_passes(lens, 147456, 16)
    assert len(plan) == 7
    assert max(sum(lens[s] for s in p) for p, _ in plan) <= 147456


def test_invalid_arguments():
    lib = L.load()
    out = (L.C.c_int32 * 4)()
    assert lib.eg2_plan_passes(L.i32_array([3, 0]), 2, 100, 0, out, None) == -1
    assert lib.eg2_plan_passes(L.i32_array([3]), 1, 0, 0, out, None) == -1
    assert lib.eg2_plan_passes(L.i32_array([3]), 1, 100, -1, out, None) == -1
    assert lib.eg2_plan_passes(L.i32_array([3]), 0, 100, 0, out, None) == 0
