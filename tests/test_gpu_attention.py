"""Attention known-answer tests after examples/check_attention.rs: the tcgen05 flash kernel
(bf16) and the f32 kernel against exact float64 attention, at tile-edge lengths, with and without
a window, logits from smooth to peaked, rows outside the sequences untouched, and packed tile lists
identical to single-sequence launches."""
import ctypes as C

import numpy as np
import pytest

from conftest import pkg
from test_oracle import exact_attention

L = pkg("lib")
W = pkg("weights")
torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

PAD_BEFORE, PAD_AFTER = 3, 2


def run_attention(kind, q, k, v, lens, nh, nkv, hd, window):
    """q/k/v for PAD_BEFORE + sum(lens) + PAD_AFTER rows; sequences start at row PAD_BEFORE.
    The padding rows are passed as a leading and a trailing sequence whose outputs are discarded,
    so the sentinel check covers rows belonging to other sequences."""
    lib = L.load()
    rows = q.shape[0]
    if kind == L.EG2_BF16:
        conv = lambda a: torch.from_numpy(W.f32_to_bf16_bits(a).view(np.int16)).cuda()
        out = torch.full((rows, nh * hd), 0x40E0, dtype=torch.int16, device="cuda")
    else:
        conv = lambda a: torch.from_numpy(a).cuda()
        out = torch.full((rows, nh * hd), 7.0, dtype=torch.float32, device="cuda")
    qd, kd, vd = conv(q), conv(k), conv(v)
    all_lens = [PAD_BEFORE] + list(lens) + [PAD_AFTER]
    rc = lib.eg2_attention(kind, C.c_void_p(qd.data_ptr()), C.c_void_p(kd.data_ptr()), C.c_void_p(vd.data_ptr()),
                           C.c_void_p(out.data_ptr()), L.i32_array(all_lens), len(all_lens), nh, nkv, hd,
                           -1 if window is None else window, None)
    torch.cuda.synchronize()
    assert rc == 0, L.ERRORS.get(rc, rc)
    o = out.cpu().numpy()
    if kind == L.EG2_BF16:
        o = W.bf16_bits_to_f32(o.view(np.uint16))
    return o


def sample(rng, rows, width, sigma, bf16):
    a = (rng.standard_normal((rows, width)) * sigma).astype(np.float32)
    return W.bf16_round(a) if bf16 else a


# Text sliding (head 256) and global (head 512) layers; the vision tower (12 heads of 64, one K/V head each).
CONFIGS = [(4, 2, 256, [None, 512, 7]), (4, 1, 512, [None, 7]), (12, 12, 64, [None, 7])]


@pytest.mark.parametrize("nh,nkv,hd,windows", CONFIGS)
def test_flash_bf16_single_sequences(nh, nkv, hd, windows):
    rng = np.random.default_rng(0x9E37)
    base = hd ** -0.25
    worst = 0.0
    for sigma in (base, 2 * base, 4 * base):
        for seq in (1, 5, 31, 32, 33, 63, 64, 65, 127, 300, 700):
            for window in windows:
                rows = PAD_BEFORE + seq + PAD_AFTER
                q, k = sample(rng, rows, nh * hd, sigma, True), sample(rng, rows, nkv * hd, sigma, True)
                v = sample(rng, rows, nkv * hd, 1.0, True)
                o = run_attention(L.EG2_BF16, q, k, v, [seq], nh, nkv, hd, window)
                inner = slice(PAD_BEFORE, PAD_BEFORE + seq)
                want = exact_attention(q[inner], k[inner], v[inner], [seq], nh, nkv, hd, window)
                got = o[inner]
                assert np.isfinite(got).all()
                rel = np.abs(got - want) / np.maximum(1.0, np.abs(want))
                worst = max(worst, float(rel.max()))
                assert rel.max() <= 2.5e-2, (sigma, seq, window, float(rel.max()))
    print(f"worst relative error {worst:.3e}")


@pytest.mark.parametrize("nh,nkv,hd,windows", CONFIGS)
def test_flash_bf16_packed_equals_single(nh, nkv, hd, windows):
    rng = np.random.default_rng(0x2545)
    lens = [1, 5, 31, 32, 33, 63, 64, 65, 130, 300] + [10 + int(rng.integers(0, 111)) for _ in range(20)]
    rows = PAD_BEFORE + sum(lens) + PAD_AFTER
    sigma = hd ** -0.25
    q, k = sample(rng, rows, nh * hd, sigma, True), sample(rng, rows, nkv * hd, sigma, True)
    v = sample(rng, rows, nkv * hd, 1.0, True)
    for window in windows:
        packed = run_attention(L.EG2_BF16, q, k, v, lens, nh, nkv, hd, window)
        off = PAD_BEFORE
        for seq in lens[:10]:
            sl = slice(off, off + seq)
            sub = np.concatenate([q[:PAD_BEFORE], q[sl], q[-PAD_AFTER:]])
            subk = np.concatenate([k[:PAD_BEFORE], k[sl], k[-PAD_AFTER:]])
            subv = np.concatenate([v[:PAD_BEFORE], v[sl], v[-PAD_AFTER:]])
            single = run_attention(L.EG2_BF16, sub, subk, subv, [seq], nh, nkv, hd, window)
            np.testing.assert_array_equal(single[PAD_BEFORE:PAD_BEFORE + seq], packed[sl])
            off += seq


@pytest.mark.parametrize("nh,nkv,hd,window", [(4, 2, 256, 512), (4, 1, 512, None), (12, 12, 64, None)])
def test_f32_attention_vs_exact(nh, nkv, hd, window):
    rng = np.random.default_rng(5)
    lens = [1, 64, 129, 600]
    rows = PAD_BEFORE + sum(lens) + PAD_AFTER
    sigma = hd ** -0.25
    q, k = sample(rng, rows, nh * hd, sigma, False), sample(rng, rows, nkv * hd, sigma, False)
    v = sample(rng, rows, nkv * hd, 1.0, False)
    o = run_attention(L.EG2_F32, q, k, v, lens, nh, nkv, hd, window)
    inner = slice(PAD_BEFORE, PAD_BEFORE + sum(lens))
    want = exact_attention(q[inner], k[inner], v[inner], lens, nh, nkv, hd, window)
    assert np.abs(o[inner] - want).max() < 2e-5


def test_flash_bf16_long_global_sequence():
    """One 2208-token global-layer sequence: every query sees all keys (35 key tiles)."""
    rng = np.random.default_rng(11)
    nh, nkv, hd, seq = 4, 1, 512, 2208
    rows = PAD_BEFORE + seq + PAD_AFTER
    sigma = hd ** -0.25
    q, k = sample(rng, rows, nh * hd, sigma, True), sample(rng, rows, nkv * hd, sigma, True)
    v = sample(rng, rows, nkv * hd, 1.0, True)
    o = run_attention(L.EG2_BF16, q, k, v, [seq], nh, nkv, hd, None)
    inner = slice(PAD_BEFORE, PAD_BEFORE + seq)
    pick = np.r_[0:40, 1000:1040, 2168:2208]
    qi = q[inner]
    full = exact_attention(qi, k[inner], v[inner], [seq], nh, nkv, hd, None)
    rel = np.abs(o[inner][pick] - full[pick]) / np.maximum(1.0, np.abs(full[pick]))
    assert rel.max() <= 2.5e-2


def exact_rows(q, k, v, start, seq, rows_, nh, nkv, hd, window):
    """Exact (float64) attention outputs of the selected query rows of one sequence starting at row
    `start`: every key of the sequence, or those within `window` of the query."""
    G = nh // nkv
    out = np.zeros((len(rows_), nh * hd))
    for n, i in enumerate(rows_):
        lo, hi = start, start + seq
        if window is not None:
            lo, hi = max(lo, i - window), min(hi, i + window + 1)
        for h in range(nh):
            g = h // G
            qi = q[i, h * hd:(h + 1) * hd].astype(np.float64)
            kk = k[lo:hi, g * hd:(g + 1) * hd].astype(np.float64)
            s = kk @ qi
            p = np.exp(s - s.max())
            out[n, h * hd:(h + 1) * hd] = (p / p.sum()) @ v[lo:hi, g * hd:(g + 1) * hd].astype(np.float64)
    return out


@pytest.mark.parametrize("window", [None, 7])
def test_flash_bf16_global_layers_in_the_four_cta_regime(window):
    """Passes of at least 8,192 rows run head 512 on clusters of four (S once per key tile, P sent to
    the CTAs that hold O): four long sequences against exact attention at their first, middle and last
    rows (with a window the sliding masks of the same kernel)."""
    rng = np.random.default_rng(23)
    nh, nkv, hd = 4, 1, 512
    lens = [2208, 2208, 2208, 1700]
    rows = PAD_BEFORE + sum(lens) + PAD_AFTER
    assert rows >= 8192
    sigma = hd ** -0.25
    q, k = sample(rng, rows, nh * hd, sigma, True), sample(rng, rows, nkv * hd, sigma, True)
    v = sample(rng, rows, nkv * hd, 1.0, True)
    o = run_attention(L.EG2_BF16, q, k, v, lens, nh, nkv, hd, window)
    assert np.isfinite(o).all()
    off = PAD_BEFORE
    worst = 0.0
    for seq in lens:
        pick = [off + i for i in list(range(0, 12)) + list(range(seq // 2, seq // 2 + 12)) + list(range(seq - 12, seq))]
        want = exact_rows(q, k, v, off, seq, pick, nh, nkv, hd, window)
        rel = np.abs(o[pick] - want) / np.maximum(1.0, np.abs(want))
        worst = max(worst, float(rel.max()))
        assert rel.max() <= 2.5e-2, (seq, float(rel.max()))
        off += seq
    print(f"worst relative error {worst:.3e}")


def test_four_cta_regime_result_independent_of_neighbours():
    """In the four-CTA regime a sequence's rows depend only on that sequence: the same bits behind
    two different sets of filler sequences."""
    rng = np.random.default_rng(31)
    nh, nkv, hd = 4, 1, 512
    sigma = hd ** -0.25
    seq = 300
    outs = []
    for fill in ([4000, 4400], [2208, 3000, 3100]):
        lens = fill + [seq]
        rows = PAD_BEFORE + sum(lens) + PAD_AFTER
        assert rows >= 8192
        q, k = sample(rng, rows, nh * hd, sigma, True), sample(rng, rows, nkv * hd, sigma, True)
        v = sample(rng, rows, nkv * hd, 1.0, True)
        outs.append((q, k, v, lens, rows))
    # The sequence itself is the same in both calls.
    base = np.random.default_rng(77)
    sq, sk = sample(base, seq, nh * hd, sigma, True), sample(base, seq, nkv * hd, sigma, True)
    sv = sample(base, seq, nkv * hd, 1.0, True)
    got = []
    for q, k, v, lens, rows in outs:
        s0 = PAD_BEFORE + sum(lens[:-1])
        q[s0:s0 + seq], k[s0:s0 + seq], v[s0:s0 + seq] = sq, sk, sv
        o = run_attention(L.EG2_BF16, q, k, v, lens, nh, nkv, hd, None)
        got.append(o[s0:s0 + seq])
    np.testing.assert_array_equal(got[0], got[1])
