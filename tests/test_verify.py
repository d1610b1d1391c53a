"""The reference's tolerance-profile unit tests (src/verify.rs:559-653), restated."""
import numpy as np

from conftest import pkg

V = pkg("verify")


def unit_vec():
    v = np.array([((i * 37 % 101) - 50.0) / 50.0 for i in range(768)], dtype=np.float32)
    return v / np.sqrt((v * v).sum())


def check(got, want, limit):
    return V.vec_check("t", got, want, limit)


def test_profile_follows_precision():
    assert V.for_precision("f32").name == "float32"
    assert V.for_precision(0).name == "float32"
    assert V.for_precision("tf32").name == "tf32"
    assert V.for_precision("bf16").name == "bf16"


def test_tf32_profile_keeps_strict_cpu_side_limits():
    f = V.FLOAT32
    for t in (V.TF32, V.BF16):
        assert (t.pixels.max_abs, t.pixels.min_cos) == (f.pixels.max_abs, f.pixels.min_cos)
        assert (t.mel.max_abs, t.mel.min_cos) == (f.mel.max_abs, f.mel.min_cos)
    assert f.embedding.max_abs == V.TOL_EMBEDDING
    assert f.soft_tokens.max_abs == V.TOL_SOFT_TOKENS


def test_float32_profile_rejects_tf32_sized_noise():
    want = unit_vec()
    got = want.copy()
    got[0] += 3.6e-4
    assert not check(got, want, V.FLOAT32.embedding).passed()
    assert check(got, want, V.TF32.embedding).passed()


def test_tf32_profile_accepts_tf32_noise_and_rejects_real_errors():
    want = unit_vec()

    def signed(d):
        return np.array([x + (d if i % 2 == 0 else -d) for i, x in enumerate(want)], dtype=np.float32)

    assert check(signed(1e-4), want, V.TF32.embedding).passed()
    c = check(signed(9e-4), want, V.TF32.embedding)
    assert c.max_abs <= V.TF32.embedding.max_abs and not c.passed()
    big = want.copy()
    big[5] += 2e-3
    assert not check(big, want, V.TF32.embedding).passed()
    assert not check(want[::-1].copy(), want, V.TF32.embedding).passed()
    soft = np.tile(want * np.sqrt(np.float32(768)), 200)
    noisy = soft.copy()
    noisy[3] += 0.1
    assert check(noisy, soft, V.TF32.soft_tokens).passed()
    flipped = np.where(np.arange(soft.size) % 16 == 0, -soft, soft)
    assert not check(flipped, soft, V.TF32.soft_tokens).passed()


def test_bf16_profile_accepts_bf16_noise_and_rejects_real_errors():
    want = unit_vec()
    noisy = np.array([x + (2e-4 if i % 2 == 0 else -2e-4) for i, x in enumerate(want)], dtype=np.float32)
    noisy[7] += 1.5e-3
    assert check(noisy, want, V.BF16.embedding).passed()
    assert not check(noisy, want, V.TF32.embedding).passed()
    assert not check(noisy, want, V.FLOAT32.embedding).passed()
    flipped = np.where(np.arange(768) % 16 == 0, -want, want)
    assert not check(flipped, want, V.BF16.embedding).passed()
    assert not check(want + 3e-3, want, V.BF16.embedding).passed()


def test_nan_and_length_mismatch_fail():
    want = unit_vec()
    got = want.copy()
    got[0] = np.nan
    assert not check(got, want, V.TF32.embedding).passed()
    assert not check(got, want, V.FLOAT32.embedding).passed()
    assert not check(want[:767], want, V.TF32.embedding).passed()
    assert not V.Check("t", 0.0, None, V.TF32.embedding).passed()


def test_id_mismatch_fails_in_every_profile():
    v = unit_vec()
    for t in (V.FLOAT32, V.TF32, V.BF16):
        assert not V.vec_check("t", v, v, t.embedding, ids_ok=False).passed()
