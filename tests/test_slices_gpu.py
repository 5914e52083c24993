"""Channel-slice outputs and strided inputs (the in-place torch.cat path).

lotus_conv2d_fwd_slice / lotus_tconv2d_fwd_slice write a producer's output
into its channel slice of a wider NHWC tensor, lotus_maxpool2d_fwd_strided
reads such a slice.  Each must equal the dense entry point bit for bit and
leave the other channels untouched; the U-Net graph with concat fusion and
memory planning must give exactly the outputs of the graph without them.
"""
import ctypes

import numpy as np
import pytest
import torch

from lotusinfer_b200 import abi
from lotusinfer_b200 import kernels as K
from lotusinfer_b200.abi import Pool2dDesc

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SENTINEL = 0x7BFF  # largest finite fp16: must survive outside the slice


def _wide(n, h, w, cs_total):
    y = torch.empty((n, h, w, cs_total), dtype=torch.int16, device=DEV)
    y.fill_(SENTINEL)
    return y.view(torch.float16)


@pytest.mark.parametrize("case", [
    # n, c, h, w, cout, k, stride, pad, act, total channels, first channel, split-K workspace
    (2, 64, 56, 56, 64, 3, 1, 1, 1, 128, 64, False),    # resident-weight halo path
    (2, 128, 28, 28, 128, 3, 1, 1, 1, 256, 0, False),   # im2col path
    (1, 256, 14, 14, 256, 3, 1, 1, 0, 512, 256, False),  # 256-column tiles
    (1, 256, 7, 7, 256, 3, 1, 1, 1, 264, 8, True),      # split-K reduction writes the slice
    (2, 32, 40, 40, 32, 3, 1, 1, 1, 96, 64, False),     # U-Net level-1 shape
])
def test_conv2d_slice_equals_dense(case):
    n, c, h, w, cout, k, s, p, act, cs_total, c0, use_ws = case
    torch.manual_seed(sum(case[:9]))
    x = K.to_nhwc(torch.randn(n, c, h, w, device=DEV))
    wp = K.conv2d_prepack(torch.randn(cout, c, k, k, device=DEV) * (2.0 / (c * k * k)) ** 0.5, c)
    b = torch.rand(cout, device=DEV) * 0.2 - 0.1
    d = K.conv_desc(n, c, h, w, cout, k, s, p, act)
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    ws_bytes = abi.lib().lotus_conv2d_workspace_bytes(ctypes.byref(d)) if use_ws else 0
    assert not use_ws or ws_bytes > 0
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=DEV)
    dense = torch.empty((n, oh, ow, abi.channel_stride(cout)), dtype=torch.float16, device=DEV)
    abi.check(abi.lib().lotus_conv2d_fwd_ws(K._ptr(x), K._ptr(wp), K._ptr(b), None, K._ptr(dense), ctypes.byref(d),
                                            K._ptr(ws) if use_ws else None, ws_bytes, K._stream()))
    y = _wide(n, oh, ow, cs_total)
    abi.check(abi.lib().lotus_conv2d_fwd_slice(K._ptr(x), K._ptr(wp), K._ptr(b), None,
                                               ctypes.c_void_p(y.data_ptr() + 2 * c0), cs_total, ctypes.byref(d),
                                               K._ptr(ws) if use_ws else None, ws_bytes, K._stream()))
    assert torch.equal(y[..., c0:c0 + cout], dense[..., :cout])
    yi = y.view(torch.int16)
    assert bool((yi[..., :c0] == SENTINEL).all()) and bool((yi[..., c0 + cout:] == SENTINEL).all())
    assert abi.device_error() == 0


def test_tconv2d_slice_and_strided_maxpool():
    n, c, h, w, cout = 2, 256, 16, 16, 128
    torch.manual_seed(3)
    x = K.to_nhwc(torch.randn(n, c, h, w, device=DEV))
    wp = K.tconv2d_prepack(torch.randn(c, cout, 2, 2, device=DEV) * (1.0 / c) ** 0.5)
    b = torch.rand(cout, device=DEV) * 0.2 - 0.1
    dense = K.tconv2d(x, c, wp, b, cout, 2, 2, 0, 0, 1)
    d = K.tconv_desc(n, c, h, w, cout, 2, 2, 0, 0, 1)
    y = _wide(n, 2 * h, 2 * w, 256)
    abi.check(abi.lib().lotus_tconv2d_fwd_slice(K._ptr(x), K._ptr(wp), K._ptr(b), ctypes.c_void_p(y.data_ptr()),
                                                256, ctypes.byref(d), K._stream()))
    assert torch.equal(y[..., :cout], dense[..., :cout])
    assert bool((y.view(torch.int16)[..., cout:] == SENTINEL).all())
    # a max pool reading the upper half of a wider tensor in place
    src = torch.randn(n, 2 * h, 2 * w, 256, device=DEV).half()
    pd = Pool2dDesc(n, 128, 2 * h, 2 * w, 2, 2, 2, 2, 0, 0, 0)
    got = torch.empty((n, h, w, 128), dtype=torch.float16, device=DEV)
    abi.check(abi.lib().lotus_maxpool2d_fwd_strided(ctypes.c_void_p(src.data_ptr() + 2 * 128), 256, K._ptr(got),
                                                    ctypes.byref(pd), K._stream()))
    want = K.maxpool2d(src[..., 128:].contiguous(), 128, 2, 2, 0)
    assert torch.equal(got, want)
    assert abi.device_error() == 0


@pytest.mark.parametrize("name,batch", [("unet", 2), ("resnet18", 4), ("alexnet", 3)])
def test_concat_fusion_and_memory_plan_keep_outputs(tmp_path, name, batch):
    from lotusinfer_b200 import synth
    from lotusinfer_b200.graph import Graph
    param, binp = synth.make_model(name, str(tmp_path), seed=0)
    x = synth.synthetic_input(name, batch, seed=6)
    g1 = Graph(param, binp, batch)
    g2 = Graph(param, binp, batch, fuse_concat=False, plan_memory=False)
    a, b = g1.run(x), g2.run(x)
    np.testing.assert_array_equal(a, b)
    types1 = [l["type"] for l in g1.layers()]
    if name == "unet":
        assert g1.launches_per_forward() == g2.launches_per_forward() - types1.count("torch.cat")
    assert g1.activation_bytes() < g2.activation_bytes()
    g1.close()
    g2.close()
