"""Pass policy on the GPU (eg2_embed_packed / eg2_forward_packed split into passes, see
eg2_plan_passes) and the bf16 parity of very short documents.

Short documents get no averaging over tokens from the mean pool, so their bf16 rounding errors reach
the embedding whole: in bf16 over 40 seeds, 2- and 3-token documents exceed the bf16 profile's 4e-3
max-abs (src/verify.rs:104-110). bf16 contexts therefore run sequences of at most 16 tokens in
TF32; the sweep below checks every length from 1 token up past that threshold, both packed into one
call and one document per call (the CUDA-graph path), against the CPU oracle.
"""
import numpy as np
import pytest

import oracle as O
from conftest import pkg
from test_gpu_text import check_embeddings

B = pkg("backend")
V = pkg("verify")
L = pkg("lib")
torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu
SWEEP_LENS = (1, 2, 3, 5, 8, 12, 16, 17, 24)
SWEEP_SEEDS = 40


def ids_of(n, seed):
    return np.random.default_rng(100_000 * n + seed).integers(0, 262144, size=n).astype(np.uint32)


@pytest.fixture(scope="module")
def sweep(oracle_text):
    seqs = [ids_of(n, s) for n in SWEEP_LENS for s in range(SWEEP_SEEDS)]
    want = np.concatenate([oracle_text.embed_ids([x]) for x in seqs], axis=0)
    return seqs, want


def _report(got, want, seqs, label):
    worst = {}
    for i, s in enumerate(seqs):
        for d in (768, 512, 256, 128):
            cut = O.truncate_and_normalize(want[i:i + 1], d)[0]
            c = V.vec_check(f"{label}[{i}]@{d}", got[d][i], cut, V.BF16.embedding)
            w = worst.setdefault(len(s), [0.0, 1.0])
            w[0] = max(w[0], c.max_abs)
            w[1] = min(w[1], c.cos)
    for n in sorted(worst):
        print(f"{label} len {n:3d}: worst max|d| {worst[n][0]:.2e} ({worst[n][0] / 4e-3:.0%} of 4e-3), "
              f"min cos {worst[n][1]:.8f}")
    return worst


def test_short_document_sweep_packed(dev_bf16, sweep):
    seqs, want = sweep
    got = B.TextBackend(dev_bf16).embed_ids(seqs)
    _report(got, want, seqs, "packed")
    check_embeddings(got, want, V.BF16, "sweep/packed")


def test_short_document_sweep_one_per_call(dev_bf16, sweep):
    seqs, want = sweep
    tb = B.TextBackend(dev_bf16)
    rows = [tb.embed_ids([x]) for x in seqs]
    got = {d: np.concatenate([r[d] for r in rows], axis=0) for d in (768, 512, 256, 128)}
    _report(got, want, seqs, "single")
    check_embeddings(got, want, V.BF16, "sweep/single")


def test_short_passes_are_the_tf32_context(dev_bf16, dev_tf32):
    """The TF32 passes of a bf16 context compute exactly what a TF32 context computes."""
    assert dev_bf16.pass_policy()[1] == 16
    seqs = [ids_of(n, 7) for n in (3, 16, 1, 9, 12)]
    a = B.TextBackend(dev_bf16).embed_ids(seqs)[768]
    b = B.TextBackend(dev_tf32).embed_ids(seqs)[768]
    np.testing.assert_array_equal(a, b)


def test_mixed_call_equals_its_passes(dev_bf16):
    lens = [3, 2208, 5, 17, 1, 700, 16, 300, 128]
    seqs = [ids_of(n, 3) for n in lens]
    tb = B.TextBackend(dev_bf16)
    whole = tb.embed_ids(seqs)
    max_rows, pmax = dev_bf16.pass_policy()
    plan = B.plan_passes(lens, max_rows, pmax)
    assert len(plan) == 2
    for idx, _ in plan:
        part = tb.embed_ids([seqs[i] for i in idx])
        for d in (768, 128):
            np.testing.assert_array_equal(whole[d][idx], part[d])
    # Per-token states through the drop-in call: the same split.
    ids = np.concatenate(seqs)
    e = tb.embed_tokens(ids)
    states = tb.forward_packed(e, lens)
    offs = np.concatenate([[0], np.cumsum(lens)])
    for idx, _ in plan:
        rows = np.concatenate([np.arange(offs[i], offs[i + 1]) for i in idx])
        part = tb.forward_packed(e[rows], [lens[i] for i in idx])
        np.testing.assert_array_equal(states[rows], part)


def test_one_million_tokens_in_a_bounded_workspace(model_dir):
    """A call of ~1 M tokens runs as passes of at most 147,456 rows: device memory grows by about one
    pass's workspace (not the ~77 GB an unsplit pass would need), and each pass's embeddings are the
    bits of that pass run as a call of its own."""
    free0 = torch.cuda.mem_get_info()[0]
    dev = B.Device(model_dir, 0, "bf16")
    try:
        lens = [2208] * 453 + [1000, 7, 1000]
        rng = np.random.default_rng(1_000_000)
        seqs = [rng.integers(0, 262144, size=n).astype(np.uint32) for n in lens]
        tb = B.TextBackend(dev)
        whole = tb.embed_ids(seqs, dims=(128,))
        used_gb = (free0 - torch.cuda.mem_get_info()[0]) / 2 ** 30
        max_rows, pmax = dev.pass_policy()
        plan = B.plan_passes(lens, max_rows, pmax)
        print(f"{sum(lens)} tokens in {len(plan)} passes of at most {max_rows} rows; device memory used {used_gb:.1f} GB")
        assert len(plan) == 8
        assert used_gb < 16.0
        for idx, _ in plan:
            part = tb.embed_ids([seqs[i] for i in idx], dims=(128,))
            np.testing.assert_array_equal(whole[768][idx], part[768])
            np.testing.assert_array_equal(whole[128][idx], part[128])
    finally:
        dev.close()


def test_forward_packed_in_several_passes(model_dir, monkeypatch):
    """forward_packed split into passes of at most 1,024 rows writes every pass's per-token states in
    their place: the same bits as each pass called alone."""
    monkeypatch.setenv("EG2_PASS_ROWS", "1024")
    dev = B.Device(model_dir, 0, "bf16")
    try:
        assert dev.pass_policy() == (1024, 16)
        lens = [700, 500, 300, 3, 5, 1200, 16, 40]
        seqs = [ids_of(n, 11) for n in lens]
        tb = B.TextBackend(dev)
        ids = np.concatenate(seqs)
        e = tb.embed_tokens(ids)
        states = tb.forward_packed(e, lens)
        plan = B.plan_passes(lens, 1024, 16)
        assert len(plan) == 5
        offs = np.concatenate([[0], np.cumsum(lens)])
        for idx, _ in plan:
            rows = np.concatenate([np.arange(offs[i], offs[i + 1]) for i in idx])
            np.testing.assert_array_equal(states[rows], tb.forward_packed(e[rows], [lens[i] for i in idx]))
        # And the device-buffer variant gives the same bits.
        e_d = torch.from_numpy(e).cuda()
        out_d = torch.empty((sum(lens), dev.embedding_dim), dtype=torch.float32, device="cuda")
        tb.forward_packed_device(e_d.data_ptr(), lens, out_d.data_ptr())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out_d.cpu().numpy(), states)
        pooled = tb.embed_ids(seqs)
        ids_d = torch.from_numpy(ids.view(np.int32)).cuda()
        out_p = torch.empty((len(lens), 768 + 512 + 256 + 128), dtype=torch.float32, device="cuda")
        tb.embed_ids_device(ids_d.data_ptr(), lens, (768, 512, 256, 128), out_p.data_ptr())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out_p.cpu().numpy()[:, :768], pooled[768])
    finally:
        dev.close()
