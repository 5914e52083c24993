"""The preprocessing oracle against OpenCV's own output of the reference's
classification-demo pipeline (tests/golden/preprocess_cv2.npz, made by
tests/golden/make_preprocess_golden.py with cv2): within one 8-bit step
before the normalisation, the difference OpenCV's 11-bit fixed-point resize
of 8-bit images allows."""
import os

import numpy as np

from oracle import oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "preprocess_cv2.npz")


def test_oracle_matches_opencv_within_one_8bit_step():
    d = np.load(GOLD)
    for name in ("down_320x240", "up_150x200"):
        got = oracle.preprocess_bgr_u8(d[name + "_bgr"])[0]
        want = d[name + "_out"]
        assert got.shape == want.shape == (3, 224, 224)
        steps = np.abs(got - want) * 255.0 * np.array(oracle.IMAGENET_STD, np.float32)[:, None, None]
        assert steps.max() <= 1.0, (name, float(steps.max()))
        assert np.mean(steps) < 0.35  # OpenCV rounds the resized value to 8 bits: ~0.25 step on average


def test_oracle_identity_resize_is_exact_normalisation():
    """With a 224x224 source, resize 224 and crop 224 the bilinear weights
    are all zero: the output is the normalised source pixel, RGB planar."""
    rng = np.random.default_rng(3)
    img = rng.integers(0, 256, (2, 224, 224, 3), dtype=np.uint8)
    got = oracle.preprocess_bgr_u8(img, resize_hw=(224, 224))
    f = img[..., ::-1].astype(np.float32) * np.float32(1 / 255)
    want = (f - np.array(oracle.IMAGENET_MEAN, np.float32)) / np.array(oracle.IMAGENET_STD, np.float32)
    np.testing.assert_allclose(got, want.transpose(0, 3, 1, 2), rtol=0, atol=1e-6)
