"""Vision tower parity (soft tokens) against the CPU oracle per profile."""
import numpy as np
import pytest

from conftest import pkg

B = pkg("backend")
V = pkg("verify")

pytestmark = pytest.mark.gpu


def image(gh, gw, seed):
    rng = np.random.default_rng(seed)
    patches = rng.random((gh * gw, 768), dtype=np.float32)
    pos = np.array([[x, y] for y in range(gh) for x in range(gw)], dtype=np.int32)
    return patches, pos


@pytest.mark.parametrize("prec", ["bf16", "tf32", "f32"])
def test_vision_soft_tokens(prec, oracle_vision, request):
    dev = request.getfixturevalue(f"dev_{prec}")
    vb = B.VisionBackend(dev)
    prof = V.for_precision(prec)
    # 576 patches: three 256-token attention tiles, the last with 64 live rows. 12 x 12 and 6 x 24
    # have the same patch count with different positions (the position tables are rebuilt), and the
    # second 24 x 24 image reuses the tables of the first.
    for gh, gw in ((12, 12), (6, 24), (6, 21), (24, 24), (24, 24)):
        patches, pos = image(gh, gw, gh * 100 + gw)
        pooled_want, soft_want = oracle_vision.encode(patches, pos, gh, gw)
        soft, pooled = vb.encode(patches, pos, gh, gw, pooled=True)
        c = V.vec_check(f"{prec} soft {gh}x{gw}", soft, soft_want, prof.soft_tokens)
        assert c.passed(), str(c)
        print(c)


def test_vision_full_size_image(dev_bf16, oracle_vision):
    """The benchmarked image size: 48 x 48 = 2,304 patches (a 768 x 768 image after the reference's
    resize), nine full 256-token attention tiles per head, 256 soft tokens."""
    vb = B.VisionBackend(dev_bf16)
    patches, pos = image(48, 48, 4848)
    _, soft_want = oracle_vision.encode(patches, pos, 48, 48)
    soft = vb.encode(patches, pos, 48, 48)
    assert soft.shape == (256, 512)
    c = V.vec_check("bf16 soft 48x48", soft, soft_want, V.for_precision("bf16").soft_tokens)
    assert c.passed(), str(c)
    print(c)


@pytest.mark.parametrize("prec", ["bf16", "f32"])
def test_vision_batch_equals_single_images(prec, request):
    """eg2_vision_encode_batch stacks the images into one pass: each image's soft tokens and pooled states
    are the bits of that image encoded alone (every kernel's result for a row depends only on that row,
    its own image's keys and its own pooling window)."""
    vb = B.VisionBackend(request.getfixturevalue(f"dev_{prec}"))
    for gh, gw, n in ((12, 12, 3), (24, 24, 5), (6, 21, 2)):
        imgs = [image(gh, gw, 7000 + 31 * i + gh)[0] for i in range(n)]
        pos = image(gh, gw, 0)[1]
        soft_b, pooled_b = vb.encode_batch(np.stack(imgs), pos, gh, gw, pooled=True)
        for i, img in enumerate(imgs):
            soft, pooled = vb.encode(img, pos, gh, gw, pooled=True)
            np.testing.assert_array_equal(soft_b[i], soft)
            np.testing.assert_array_equal(pooled_b[i], pooled)


def test_vision_batch_parity(dev_bf16, oracle_vision):
    """Eight full-size images (48 x 48 patches) in one call, each against the oracle."""
    vb = B.VisionBackend(dev_bf16)
    imgs = [image(48, 48, 900 + i)[0] for i in range(8)]
    pos = image(48, 48, 0)[1]
    soft = vb.encode_batch(np.stack(imgs), pos, 48, 48)
    for i in (0, 7):
        _, want = oracle_vision.encode(imgs[i], pos, 48, 48)
        c = V.vec_check(f"bf16 batch soft [{i}]", soft[i], want, V.for_precision("bf16").soft_tokens)
        assert c.passed(), str(c)
        print(c)
