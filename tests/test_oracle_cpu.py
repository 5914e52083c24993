"""CPU checks of the oracle: hand-computed known answers, the reference tests'
own deterministic inputs, the reference tests' shapes, and torch CPU as an
independent second opinion (torch is a test dependency only)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle
from tests._metrics import max_abs, rel_l2


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def test_conv2d_known_answer():
    # 1x1x3x3 input, 2x2 kernel of ones, stride 1, pad 0: window sums.
    x = np.arange(9, dtype=np.float32).reshape(1, 1, 3, 3)
    w = np.ones((1, 1, 2, 2), np.float32)
    y = oracle.conv2d(x, w, np.array([0.5], np.float32))
    np.testing.assert_array_equal(y[0, 0], np.array([[8.5, 12.5], [20.5, 24.5]], np.float32))
    # padding 1 adds zero border; ReLU clamps negatives
    y2 = oracle.conv2d(-x, w, None, pad=(1, 1), act=1)
    assert y2.shape == (1, 1, 4, 4) and np.all(y2 == 0)


@pytest.mark.parametrize("shape", [
    # (n, c, h, w, cout, k, stride, pad) -- includes the reference test's 7x7 s2 Cout=17 case (smaller image)
    (1, 64, 56, 56, 64, 3, 1, 1),
    (2, 3, 61, 61, 17, 7, 2, 1),
    (1, 16, 14, 14, 32, 1, 2, 0),
    (2, 8, 9, 11, 5, 5, 3, 2),
])
def test_conv2d_vs_torch(shape):
    n, c, h, w, cout, k, s, p = shape
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / (c * k * k)), (cout, c, k, k)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    res_shape = F.conv2d(_t(x), _t(wt), _t(b), s, p).shape
    r = rng.normal(0, 1, res_shape).astype(np.float32)
    for act in (0, 1, 2):
        y = oracle.conv2d(x, wt, b, (s, s), (p, p), act, residual=r)
        ref = F.conv2d(_t(x), _t(wt), _t(b), s, p) + _t(r)
        ref = {0: ref, 1: torch.relu(ref), 2: torch.sigmoid(ref)}[act].numpy()
        assert max_abs(y, ref) < 1e-4 and rel_l2(y, ref) < 1e-5


def test_tconv2d_vs_torch():
    rng = np.random.default_rng(1)
    # reference test shape (16 -> 8 channels, 64x64, k2 s3) and U-Net's k2 s2, plus overlap/crop/output_padding
    cases = [(1, 16, 64, 64, 8, 2, 3, 0, 0), (2, 32, 8, 8, 16, 2, 2, 0, 0), (1, 8, 7, 5, 4, 3, 2, 1, 1),
             (1, 4, 6, 6, 3, 4, 2, 1, 0)]
    for n, cin, h, w, cout, k, s, p, op in cases:
        x = rng.integers(-10, 10, (n, cin, h, w)).astype(np.float32)
        wt = rng.integers(-10, 10, (cin, cout, k, k)).astype(np.float32)
        b = rng.integers(-10, 10, cout).astype(np.float32)
        y = oracle.tconv2d(x, wt, b, (s, s), (p, p), (op, op))
        ref = F.conv_transpose2d(_t(x).double(), _t(wt).double(), _t(b).double(), s, p, op).numpy()
        np.testing.assert_array_equal(y, ref.astype(np.float32))  # integer data: exact


def test_gemm_reference_formula_inputs():
    # test/test_gemm.cu:13-48 deterministic inputs (rows/cols 0 divide by zero there; start at 1)
    seq = inf = outf = 255
    i = np.arange(seq)[:, None].astype(np.float64)
    j = np.arange(inf)[None, :].astype(np.float64)
    with np.errstate(all="ignore"):
        a = np.where((i * j) % 2 == 0, -1.0 / j + 100.0 / i, 1.0 / j - 100.0 / i)
        i2 = np.arange(outf)[:, None].astype(np.float64)
        wt = np.where((i2 * j) % 2 == 0, 1.0 / j - 50.0 / i2, -1.0 / j + 50.0 / i2)
    bias = np.where(np.arange(outf) % 2 == 0, 1.0, -1.0)
    a, wt = a[1:, 1:].astype(np.float32), wt[1:, 1:].astype(np.float32)
    bias = bias[1:].astype(np.float32)
    got = oracle.gemm(a, wt, bias)
    want = a.astype(np.float64) @ wt.astype(np.float64).T + bias
    assert rel_l2(got, want) < 1e-6


def test_gemv_and_gemm_vs_numpy():
    rng = np.random.default_rng(2)
    wt = rng.normal(0, np.sqrt(1 / 512), (1000, 512)).astype(np.float32)
    x = rng.uniform(-1, 1, (3, 512)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, 1000).astype(np.float32)
    want = x.astype(np.float64) @ wt.T.astype(np.float64) + b
    assert max_abs(oracle.gemv(wt, x, b), want) < 1e-5
    assert max_abs(oracle.gemm(x, wt, b), want) < 1e-5
    assert np.all(oracle.gemm(x, wt, b, act=1) >= 0)


def test_maxpool_vs_torch_and_reference_zero_pad():
    rng = np.random.default_rng(3)
    # reference test: 257x257 C3, k9 s2 p4, non-negative ints (zero pad == -inf pad there)
    x = rng.integers(0, 100, (1, 3, 257, 257)).astype(np.float32)
    y = oracle.maxpool2d(x, (9, 9), (2, 2), (4, 4))
    np.testing.assert_array_equal(y, F.max_pool2d(_t(x), 9, 2, 4).numpy())
    np.testing.assert_array_equal(y, oracle.maxpool2d(x, (9, 9), (2, 2), (4, 4), zero_pad=True))
    # signed inputs: -inf padding (PyTorch), which the zero-padded variant does not match
    xs = rng.normal(0, 1, (2, 5, 112, 112)).astype(np.float32) - 3.0
    ys = oracle.maxpool2d(xs, (3, 3), (2, 2), (1, 1))
    np.testing.assert_array_equal(ys, F.max_pool2d(_t(xs), 3, 2, 1).numpy())
    assert not np.array_equal(ys, oracle.maxpool2d(xs, (3, 3), (2, 2), (1, 1), zero_pad=True))


def test_adaptive_avgpool_vs_torch():
    rng = np.random.default_rng(4)
    for shape, out in [((2, 16, 7, 7), (1, 1)), ((1, 3, 257, 257), (64, 64)), ((1, 8, 6, 6), (6, 6)),
                       ((1, 4, 13, 9), (6, 4))]:
        x = rng.normal(0, 1, shape).astype(np.float32)
        y = oracle.adaptive_avgpool2d(x, out)
        assert max_abs(y, F.adaptive_avg_pool2d(_t(x), out).numpy()) < 1e-5


def test_reference_avgpool_windows_agree_for_resnet_only():
    rng = np.random.default_rng(5)
    x7 = rng.normal(0, 1, (4, 7, 7)).astype(np.float32)
    assert max_abs(oracle.avgpool_reference_windows(x7, (1, 1)), x7.mean(axis=(1, 2), keepdims=True)) < 1e-6
    # AlexNet 6x6 -> 6x6: the reference's integer stride is 0, every output is x[c,0,0]
    x6 = rng.normal(0, 1, (2, 6, 6)).astype(np.float32)
    ref_win = oracle.avgpool_reference_windows(x6, (6, 6))
    assert np.allclose(ref_win, x6[:, :1, :1]) and not np.allclose(ref_win, x6)


def test_add_and_concat():
    rng = np.random.default_rng(6)
    a = rng.normal(0, 1, (2, 3, 4, 5)).astype(np.float32)
    b = rng.normal(0, 1, (2, 3, 4, 5)).astype(np.float32)
    np.testing.assert_array_equal(oracle.add(a, b), a + b)
    np.testing.assert_array_equal(oracle.add(a, b, 1), np.maximum(a + b, 0))
    c = rng.normal(0, 1, (2, 7, 4, 5)).astype(np.float32)
    np.testing.assert_array_equal(oracle.concat(a, c), np.concatenate([a, c], 1))
