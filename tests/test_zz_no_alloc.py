"""lotus_conv2d_fwd_noalloc, the conv entry point for callers that cannot
allocate device memory (a serving loop that must not trigger the device
synchronisation or the out-of-memory failure a cudaMalloc can bring, or a host
framework that owns the device memory pool).  Its split-K partial sums live in
a fixed 8 MiB scratch compiled into the library instead of a caller workspace.

Kept in its own file, collected after every other test file, so that a run
stopping at the first failure has run everything else first.  It passes on
its own in a fresh process and after the other tests (the scratch is fully
rewritten by every call).
"""
import ctypes
import zlib

import numpy as np
import pytest
import torch

from tests._metrics import assert_close

pytestmark = pytest.mark.gpu

DEV = "cuda:0"

CASES = [
    # id, n, c, h, w, cout, k, stride, pad, act, residual
    ("stage4_bs1_residual_splits", 1, 512, 7, 7, 512, 3, 1, 1, 1, True),
    ("stage3_bs1_gather_splits", 1, 256, 14, 14, 256, 3, 1, 1, 0, False),
    ("cout17_sigmoid_splits", 1, 64, 16, 16, 17, 3, 1, 1, 2, False),
    ("stage1_bs2_no_split", 2, 64, 56, 56, 64, 3, 1, 1, 1, False),
]


def _conv_noalloc(K, abi, x, c, wp, b, cout, k, s, p, act, res):
    n, h, w, _ = x.shape
    d = K.conv_desc(n, c, h, w, cout, k, s, p, act, K.OUT_NHWC_F16)
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    y = torch.empty((n, oh, ow, K.channel_stride(cout)), dtype=torch.float16, device=DEV)
    status = abi.lib().lotus_conv2d_fwd_noalloc(K._ptr(x), K._ptr(wp), K._ptr(b), K._ptr(res), K._ptr(y),
                                                ctypes.byref(d), K._stream())
    abi.check(status)
    return y


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_noalloc_matches_conv2d_fwd_on_two_calls(case):
    from lotusinfer_b200 import abi
    from lotusinfer_b200 import kernels as K
    _, n, c, h, w, cout, k, s, p, act, with_res = case
    g = torch.Generator(device=DEV).manual_seed(zlib.crc32(case[0].encode()))
    x = K.to_nhwc(torch.rand((n, c, h, w), device=DEV, generator=g) * 2 - 1)
    wt = torch.randn((cout, c, k, k), device=DEV, generator=g) * (2.0 / (c * k * k)) ** 0.5
    b = torch.rand(cout, device=DEV, generator=g) * 0.2 - 0.1
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    res = K.to_nhwc(torch.randn((n, cout, oh, ow), device=DEV, generator=g)) if with_res else None
    wp = K.conv2d_prepack(wt, c)
    want = K.from_nhwc(K.conv2d(x, c, wp, b, cout, k, s, p, act, residual=res), cout).cpu().numpy()
    first = _conv_noalloc(K, abi, x, c, wp, b, cout, k, s, p, act, res)
    second = _conv_noalloc(K, abi, x, c, wp, b, cout, k, s, p, act, res)
    for i, y in enumerate((first, second)):
        assert_close(K.from_nhwc(y, cout).cpu().numpy(), want, what=f"{case[0]} call {i + 1}")
        if y.shape[-1] != cout:
            assert torch.count_nonzero(y[..., cout:]).item() == 0
    assert torch.equal(first, second)
    assert abi.device_error() == 0


def test_noalloc_rejects_a_split_above_its_scratch():
    """A shape whose split-K would need more than the 8 MiB built in is refused
    with a clear error instead of running."""
    from lotusinfer_b200 import abi
    from lotusinfer_b200 import kernels as K
    n, c, h, w, cout, k = 1, 512, 7, 7, 2048, 3
    assert K.conv2d_workspace_bytes(n, c, h, w, cout, k, 1, 1) > (8 << 20)
    x = torch.zeros((n, h, w, K.channel_stride(c)), dtype=torch.float16, device=DEV)
    wp = torch.zeros((cout, 9 * c), dtype=torch.float16, device=DEV)
    y = torch.empty((n, h, w, K.channel_stride(cout)), dtype=torch.float16, device=DEV)
    d = K.conv_desc(n, c, h, w, cout, k, 1, 1, 0, K.OUT_NHWC_F16)
    status = abi.lib().lotus_conv2d_fwd_noalloc(K._ptr(x), K._ptr(wp), None, None, K._ptr(y), ctypes.byref(d),
                                                K._stream())
    assert status == -2  # LOTUS_ERR_UNSUPPORTED
    assert b"scratch" in abi.lib().lotus_last_error_string()
