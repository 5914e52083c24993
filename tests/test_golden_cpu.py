"""The CPU oracle against golden outputs of the reference's own operator
kernels (tests/golden/ref_ops.npz, generated on a GPU by
tests/golden/make_golden.py from the reference sources).  Integer-valued and
fp16-exact cases must match bit for bit; the others within fp32 summation
order (1e-5)."""
import os

import numpy as np
import pytest

from oracle import oracle

FIX = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_ops.npz")


@pytest.fixture(scope="module")
def gold():
    assert os.path.exists(FIX), "golden fixture missing: run tests/golden/make_golden.py on a GPU"
    return dict(np.load(FIX))


def _names(g, prefix):
    return sorted({k.split("/")[0] for k in g if k.startswith(prefix)})


def test_fixture_covers_every_operator(gold):
    for prefix in ("conv_", "tconv_", "maxpool_", "aap_", "add_", "gemm", "gemv"):
        assert _names(gold, prefix), prefix


def test_conv2d_matches_reference_kernel(gold):
    for name in _names(gold, "conv_"):
        x, w, b, y = gold[f"{name}/x"], gold[f"{name}/w"], gold[f"{name}/b"], gold[f"{name}/y"]
        s, p, act = (int(v) for v in gold[f"{name}/cfg"])
        got = oracle.conv2d(x, w, b, (s, s), (p, p), act)
        if np.all(x == np.round(x)) and np.all(w == np.round(w)):
            np.testing.assert_array_equal(got, y, err_msg=name)
        else:
            np.testing.assert_allclose(got, y, rtol=1e-5, atol=1e-5, err_msg=name)


def test_tconv2d_matches_reference_kernel(gold):
    for name in _names(gold, "tconv_"):
        x, w, b, y = gold[f"{name}/x"], gold[f"{name}/w"], gold[f"{name}/b"], gold[f"{name}/y"]
        s, act = (int(v) for v in gold[f"{name}/cfg"])
        np.testing.assert_array_equal(oracle.tconv2d(x, w, b, (s, s), (0, 0), (0, 0), act), y, err_msg=name)


def test_pooling_and_add_match_reference_kernels(gold):
    for name in _names(gold, "maxpool_"):
        k, s, act = (int(v) for v in gold[f"{name}/cfg"])
        np.testing.assert_array_equal(oracle.maxpool2d(gold[f"{name}/x"], (k, k), (s, s), (0, 0), act),
                                      gold[f"{name}/y"], err_msg=name)
    x, y = gold["aap_7to1/x"], gold["aap_7to1/y"]
    np.testing.assert_allclose(oracle.adaptive_avgpool2d(x, (1, 1)), y, rtol=1e-6, atol=1e-6)
    x, y = gold["aap_refwin_33to8/x"], gold["aap_refwin_33to8/y"]
    got = np.stack([oracle.avgpool_reference_windows(x[i], (8, 8)) for i in range(x.shape[0])])
    np.testing.assert_allclose(got, y, rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(oracle.add(gold["add_relu/a"], gold["add_relu/b"], 1), gold["add_relu/y"])


def test_gemm_and_gemv_match_reference_kernels(gold):
    np.testing.assert_array_equal(oracle.gemm(gold["gemm/a"], gold["gemm/w"], gold["gemm/b"]), gold["gemm/y"])
    got = oracle.gemv(gold["gemv/w"], gold["gemv/x"], gold["gemv/b"])[0]
    np.testing.assert_allclose(got, gold["gemv/y"], rtol=1e-5, atol=1e-5)
