"""CPU checks of the C ABI surface: the library loads, exports every entry
point include/*.h declares, and rejects invalid arguments with a status code
and message before touching the device."""
import ctypes
import os
import re

import pytest

from lotusinfer_b200 import abi
from lotusinfer_b200.abi import Conv2dDesc, Pool2dDesc, TConv2dDesc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            txt = open(os.path.join(inc, f)).read()
            txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
            names |= set(re.findall(r"\b(lotus_\w+)\s*\(", txt))
    return names


def test_library_exports_every_declared_symbol():
    L = abi.lib()
    missing = [n for n in sorted(_declared()) if not hasattr(L, n)]
    assert not missing, missing
    assert len(_declared()) >= 20


def test_python_binding_covers_ops_header():
    txt = open(os.path.join(ROOT, "include", "lotus_ops.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    for n in set(re.findall(r"\b(lotus_\w+)\s*\(", txt)):
        assert n in abi.SIGNATURES, n


def test_shape_helpers():
    L = abi.lib()
    assert L.lotus_channel_stride(3) == 8 and L.lotus_channel_stride(64) == 64 and L.lotus_channel_stride(17) == 24
    d = Conv2dDesc(256, 3, 224, 224, 64, 7, 7, 2, 2, 3, 3, 1, 0)
    oh, ow = ctypes.c_int(), ctypes.c_int()
    assert L.lotus_conv2d_out_hw(ctypes.byref(d), ctypes.byref(oh), ctypes.byref(ow)) == 0
    assert (oh.value, ow.value) == (112, 112)
    # K = 7*7*8 = 392 -> padded to 448 fp16 per output channel
    assert L.lotus_conv2d_packed_weight_bytes(ctypes.byref(d)) == 64 * 448 * 2
    t = TConv2dDesc(1, 512, 16, 16, 256, 2, 2, 2, 2, 0, 0, 0, 0, 0)
    assert L.lotus_tconv2d_out_hw(ctypes.byref(t), ctypes.byref(oh), ctypes.byref(ow)) == 0
    assert (oh.value, ow.value) == (32, 32)
    t2 = TConv2dDesc(1, 16, 64, 64, 8, 2, 2, 3, 3, 0, 0, 0, 0, 0)  # reference test: (64-1)*3+2 = 191
    assert L.lotus_tconv2d_out_hw(ctypes.byref(t2), ctypes.byref(oh), ctypes.byref(ow)) == 0
    assert (oh.value, ow.value) == (191, 191)
    p = Pool2dDesc(1, 64, 112, 112, 3, 3, 2, 2, 1, 1, 0)
    assert L.lotus_maxpool2d_out_hw(ctypes.byref(p), ctypes.byref(oh), ctypes.byref(ow)) == 0
    assert (oh.value, ow.value) == (56, 56)
    assert L.lotus_linear_packed_weight_bytes(512, 1000) == 1000 * 512 * 2
    assert L.lotus_linear_packed_weight_bytes(9216, 4096) == 4096 * 9216 * 2


@pytest.mark.parametrize("fields", [
    (0, 3, 8, 8, 4, 3, 3, 1, 1, 1, 1, 0, 0),   # n = 0
    (1, 3, 8, 8, 4, 3, 3, 0, 1, 1, 1, 0, 0),   # stride 0
    (1, 3, 2, 2, 4, 5, 5, 1, 1, 0, 0, 0, 0),   # kernel larger than input
    (1, 3, 8, 8, 4, 3, 3, 1, 1, 1, 1, 7, 0),   # unknown activation
    (1, 3, 8, 8, 4, 3, 3, 1, 1, -1, 1, 0, 0),  # negative padding
])
def test_conv_rejects_bad_descriptors(fields):
    L = abi.lib()
    d = Conv2dDesc(*fields)
    assert L.lotus_conv2d_out_hw(ctypes.byref(d), None, None) == -1
    assert abi.last_error().startswith("conv2d")


def test_entry_points_reject_null_and_misaligned_pointers_before_launch():
    L = abi.lib()
    d = Conv2dDesc(1, 64, 8, 8, 64, 3, 3, 1, 1, 1, 1, 1, 0)
    assert L.lotus_conv2d_fwd(None, None, None, None, None, ctypes.byref(d), None) == -1
    assert "null" in abi.last_error()
    assert L.lotus_conv2d_fwd(ctypes.c_void_p(0x1008), ctypes.c_void_p(0x2000), None, None,
                              ctypes.c_void_p(0x3000), ctypes.byref(d), None) == -1
    assert "aligned" in abi.last_error()
    assert L.lotus_gemv_bias_fwd(ctypes.c_void_p(16), 0, ctypes.c_void_p(16), 0, None, ctypes.c_void_p(16), 0,
                                 9, 10, 10, 0, None) == -1   # batch > 8
    assert L.lotus_add_act_fwd(None, None, None, 10, 8, 0, None) == -1
    p = Pool2dDesc(1, 8, 8, 8, 3, 3, 2, 2, 2, 2, 0)      # padding > kernel/2
    assert L.lotus_maxpool2d_fwd(ctypes.c_void_p(16), ctypes.c_void_p(32), ctypes.byref(p), None) == -1
    t = TConv2dDesc(1, 8, 4, 4, 8, 2, 2, 2, 2, 0, 0, 2, 0, 0)  # output_padding >= stride
    assert L.lotus_tconv2d_out_hw(ctypes.byref(t), None, None) == -1
    assert L.lotus_linear_prepack(None, None, 4, 4, 0, 0, 0, None) == -1
    assert L.lotus_linear_prepack(ctypes.c_void_p(16), ctypes.c_void_p(16), 10, 4, 2, 2, 2, None) == -1  # 2*2*2 != 10


def test_splitk_workspace_queries():
    """The split-K planner needs no GPU: small grids with long K ask for a
    workspace, full grids and the GEMV path do not."""
    from lotusinfer_b200 import kernels as K
    assert K.conv2d_workspace_bytes(1, 512, 7, 7, 512, 3, 1, 1) > 0      # 4 output tiles, K = 4608
    assert K.conv2d_workspace_bytes(256, 512, 7, 7, 512, 3, 1, 1) == 0   # 196 tiles fill the GPU
    assert K.conv2d_workspace_bytes(1, 3, 20, 20, 8, 3, 1, 1) == 0       # K = 64: one K block
    # the max query adds the pair kernel's last-wave split, which needs the
    # device's resident-pair count: without a GPU it equals the split-K need
    for shape in [(1, 512, 7, 7, 512, 3, 1, 1), (256, 512, 7, 7, 512, 3, 1, 1), (2, 64, 20, 20, 64, 3, 1, 1)]:
        assert K.conv2d_workspace_bytes(*shape, use_max=True) >= K.conv2d_workspace_bytes(*shape)
    L = abi.lib()
    assert L.lotus_linear_workspace_bytes(32, 9216, 4096) > 0
    assert L.lotus_linear_workspace_bytes(4, 9216, 4096) == 0            # batch <= 8 runs the GEMV


def test_conv2d_maxpool_support_query():
    """The fused conv + pool entry point says which shapes it takes, without a GPU."""
    from lotusinfer_b200 import abi
    from lotusinfer_b200.abi import Conv2dDesc, Pool2dDesc
    L = abi.lib()
    ok = Conv2dDesc(256, 12, 115, 115, 64, 4, 4, 1, 1, 0, 0, 1, 0)
    pool = Pool2dDesc(256, 64, 112, 112, 3, 3, 2, 2, 1, 1, 0)
    assert L.lotus_conv2d_maxpool_supported(ctypes.byref(ok), ctypes.byref(pool)) == 0
    assert L.lotus_conv2d_maxpool_supported(ctypes.byref(ok), None) == 0
    padded = Conv2dDesc(1, 64, 56, 56, 64, 3, 3, 1, 1, 1, 1, 1, 0)
    assert L.lotus_conv2d_maxpool_supported(ctypes.byref(padded), None) == -2
    wide = Conv2dDesc(1, 12, 200, 200, 64, 4, 4, 1, 1, 0, 0, 1, 0)  # 197-pixel output rows
    assert L.lotus_conv2d_maxpool_supported(ctypes.byref(wide), None) == -2
    cout128 = Conv2dDesc(1, 12, 115, 115, 128, 4, 4, 1, 1, 0, 0, 1, 0)
    assert L.lotus_conv2d_maxpool_supported(ctypes.byref(cout128), None) == -2
    pool2 = Pool2dDesc(256, 64, 112, 112, 2, 2, 2, 2, 0, 0, 0)
    assert L.lotus_conv2d_maxpool_supported(ctypes.byref(ok), ctypes.byref(pool2)) == -2
    wrong_in = Pool2dDesc(256, 64, 111, 112, 3, 3, 2, 2, 1, 1, 0)
    assert L.lotus_conv2d_maxpool_supported(ctypes.byref(ok), ctypes.byref(wrong_in)) == -1
    # with the pool, conv rows up to 120 pixels (60 pooled columns, 15 per TMEM lane quarter)
    for ow, want in ((120, 0), (121, -2), (128, -2)):
        c = Conv2dDesc(2, 12, 40, ow + 3, 64, 4, 4, 1, 1, 0, 0, 1, 0)
        pl = Pool2dDesc(2, 64, 37, ow, 3, 3, 2, 2, 1, 1, 0)
        assert L.lotus_conv2d_maxpool_supported(ctypes.byref(c), ctypes.byref(pl)) == want, ow
        assert L.lotus_conv2d_maxpool_supported(ctypes.byref(c), None) == 0, ow
