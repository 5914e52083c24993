"""Per-operator calls through the C ABI on torch-owned device memory.

Activations are NHWC fp16 tensors of shape [N, H, W, Cs] with Cs the channel
count rounded up to 8 (pad channels zero).  Each function allocates its output
with torch, then calls the matching ``lotus_*`` entry point on the current
torch stream.  These mirror the reference's operator signatures
(include/operator/*.cuh) one call per layer instead of one per sample.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Tuple

import torch

from . import abi
from .abi import ACT_NONE, OUT_NHWC_F16, OUT_ROWS_F32, Conv2dDesc, Pool2dDesc, TConv2dDesc, check, channel_stride


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream: Optional[torch.cuda.Stream] = None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _pair(v) -> Tuple[int, int]:
    return (v, v) if isinstance(v, int) else (int(v[0]), int(v[1]))


# --------------------------------------------------------------------- layout
def to_nhwc(x: torch.Tensor) -> torch.Tensor:
    """NCHW fp32 (cuda) -> NHWC fp16 [N, H, W, Cs]."""
    assert x.is_cuda and x.dtype == torch.float32 and x.dim() == 4
    x = x.contiguous()
    n, c, h, w = x.shape
    y = torch.empty((n, h, w, channel_stride(c)), dtype=torch.float16, device=x.device)
    check(abi.lib().lotus_nchw_f32_to_nhwc_f16(_ptr(x), _ptr(y), n, c, h, w, _stream()))
    return y


def space_to_depth(x: torch.Tensor, factor: int, pad: int, out_hw) -> torch.Tensor:
    """NCHW fp32 (cuda) -> NHWC fp16 [N, OH, OW, Cs(C*f*f)] space-to-depth of the padded image."""
    x = x.contiguous()
    n, c, h, w = x.shape
    oh, ow = out_hw
    y = torch.empty((n, oh, ow, channel_stride(c * factor * factor)), dtype=torch.float16, device=x.device)
    check(abi.lib().lotus_space_to_depth_f16(_ptr(x), _ptr(y), n, c, h, w, factor, pad, pad, oh, ow, _stream()))
    return y


def from_nhwc(y: torch.Tensor, c: int) -> torch.Tensor:
    """NHWC fp16 [N, H, W, Cs] -> NCHW fp32 with c channels."""
    n, h, w, cs = y.shape
    assert cs == channel_stride(c)
    out = torch.empty((n, c, h, w), dtype=torch.float32, device=y.device)
    check(abi.lib().lotus_nhwc_f16_to_nchw_f32(_ptr(y), _ptr(out), n, c, h, w, _stream()))
    return out


# --------------------------------------------------------------------- conv
def conv_desc(n, c_in, h, w, c_out, k, stride=1, pad=0, act=ACT_NONE, out_kind=OUT_NHWC_F16) -> Conv2dDesc:
    kh, kw = _pair(k)
    sh, sw = _pair(stride)
    ph, pw = _pair(pad)
    return Conv2dDesc(n, c_in, h, w, c_out, kh, kw, sh, sw, ph, pw, act, out_kind)


def conv2d_prepack(w_oihw: torch.Tensor, c_in: int) -> torch.Tensor:
    """OIHW fp32 weights -> packed fp16 [Cout, K_pad]."""
    cout, cin, kh, kw = w_oihw.shape
    assert cin == c_in
    d = conv_desc(1, c_in, kh, kw, cout, (kh, kw))
    nbytes = abi.lib().lotus_conv2d_packed_weight_bytes(ctypes.byref(d))
    out = torch.empty(nbytes // 2, dtype=torch.float16, device=w_oihw.device)
    check(abi.lib().lotus_conv2d_prepack(_ptr(w_oihw.contiguous().float()), _ptr(out), ctypes.byref(d), _stream()))
    return out.view(cout, -1)


def conv2d_workspace_bytes(n, c_in, h, w, c_out, k, stride=1, pad=0, act=ACT_NONE, out_f32=False,
                           use_max=False) -> int:
    """Workspace bytes the split-K plan of this conv wants (0 = no split);
    use_max: also the pair-tile kernel's optional last-wave split."""
    d = conv_desc(n, c_in, h, w, c_out, k, stride, pad, act, OUT_ROWS_F32 if out_f32 else OUT_NHWC_F16)
    fn = abi.lib().lotus_conv2d_workspace_bytes_max if use_max else abi.lib().lotus_conv2d_workspace_bytes
    return int(fn(ctypes.byref(d)))


def conv2d(x: torch.Tensor, c_in: int, w_packed: torch.Tensor, bias: Optional[torch.Tensor], c_out: int,
           k, stride=1, pad=0, act=ACT_NONE, residual: Optional[torch.Tensor] = None,
           out_f32: bool = False, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """NHWC fp16 conv2d; returns NHWC fp16 [N, OH, OW, Cs_out] or fp32 rows [N*OH*OW, Cout].
    With `workspace` (a device buffer) the call may split K (lotus_conv2d_fwd_ws)."""
    n, h, w, cs = x.shape
    assert cs == channel_stride(c_in)
    d = conv_desc(n, c_in, h, w, c_out, k, stride, pad, act, OUT_ROWS_F32 if out_f32 else OUT_NHWC_F16)
    oh, ow = ctypes.c_int(), ctypes.c_int()
    check(abi.lib().lotus_conv2d_out_hw(ctypes.byref(d), ctypes.byref(oh), ctypes.byref(ow)))
    if out_f32:
        y = torch.empty((n * oh.value * ow.value, c_out), dtype=torch.float32, device=x.device)
    else:
        y = torch.empty((n, oh.value, ow.value, channel_stride(c_out)), dtype=torch.float16, device=x.device)
    if workspace is None:
        check(abi.lib().lotus_conv2d_fwd(_ptr(x), _ptr(w_packed), _ptr(bias), _ptr(residual), _ptr(y),
                                         ctypes.byref(d), _stream()))
    else:
        check(abi.lib().lotus_conv2d_fwd_ws(_ptr(x), _ptr(w_packed), _ptr(bias), _ptr(residual), _ptr(y),
                                            ctypes.byref(d), _ptr(workspace),
                                            workspace.numel() * workspace.element_size(), _stream()))
    return y


# --------------------------------------------------------------------- tconv
def tconv_desc(n, c_in, h, w, c_out, k, stride=2, pad=0, out_pad=0, act=ACT_NONE) -> TConv2dDesc:
    kh, kw = _pair(k)
    sh, sw = _pair(stride)
    ph, pw = _pair(pad)
    oph, opw = _pair(out_pad)
    return TConv2dDesc(n, c_in, h, w, c_out, kh, kw, sh, sw, ph, pw, oph, opw, act)


def tconv2d_prepack(w_iokk: torch.Tensor, stride=2) -> torch.Tensor:
    cin, cout, kh, kw = w_iokk.shape
    d = tconv_desc(1, cin, 4, 4, cout, (kh, kw), stride)
    nbytes = abi.lib().lotus_tconv2d_packed_weight_bytes(ctypes.byref(d))
    out = torch.empty(nbytes // 2, dtype=torch.float16, device=w_iokk.device)
    check(abi.lib().lotus_tconv2d_prepack(_ptr(w_iokk.contiguous().float()), _ptr(out), ctypes.byref(d), _stream()))
    return out


def tconv2d(x: torch.Tensor, c_in: int, w_packed: torch.Tensor, bias: Optional[torch.Tensor], c_out: int, k,
            stride=2, pad=0, out_pad=0, act=ACT_NONE) -> torch.Tensor:
    n, h, w, cs = x.shape
    d = tconv_desc(n, c_in, h, w, c_out, k, stride, pad, out_pad, act)
    oh, ow = ctypes.c_int(), ctypes.c_int()
    check(abi.lib().lotus_tconv2d_out_hw(ctypes.byref(d), ctypes.byref(oh), ctypes.byref(ow)))
    y = torch.empty((n, oh.value, ow.value, channel_stride(c_out)), dtype=torch.float16, device=x.device)
    check(abi.lib().lotus_tconv2d_fwd(_ptr(x), _ptr(w_packed), _ptr(bias), _ptr(y), ctypes.byref(d), _stream()))
    return y


# --------------------------------------------------------------------- linear
def linear_prepack(w: torch.Tensor, fc_chw: Optional[Sequence[int]] = None) -> torch.Tensor:
    out_f, in_f = w.shape
    nbytes = abi.lib().lotus_linear_packed_weight_bytes(in_f, out_f)
    out = torch.empty(nbytes // 2, dtype=torch.float16, device=w.device)
    c, h, ww = fc_chw if fc_chw is not None else (0, 0, 0)
    check(abi.lib().lotus_linear_prepack(_ptr(w.contiguous().float()), _ptr(out), in_f, out_f, c, h, ww, _stream()))
    return out.view(out_f, -1)


def linear(x: torch.Tensor, w_packed: torch.Tensor, bias: Optional[torch.Tensor], in_f: int, out_f: int,
           act=ACT_NONE, out_f32=True, force_gemm=False, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x fp16 rows [M, Cs(in_f)] -> fp32 [M, out_f] or fp16 [M, Cs(out_f)].
    With `workspace` the GEMM path may split K (lotus_linear_fwd_ws)."""
    m = x.shape[0]
    if out_f32:
        y = torch.empty((m, out_f), dtype=torch.float32, device=x.device)
    else:
        y = torch.empty((m, channel_stride(out_f)), dtype=torch.float16, device=x.device)
    if workspace is not None:
        check(abi.lib().lotus_linear_fwd_ws(_ptr(x), _ptr(w_packed), _ptr(bias), _ptr(y), m, in_f, out_f, act,
                                            OUT_ROWS_F32 if out_f32 else OUT_NHWC_F16, _ptr(workspace),
                                            workspace.numel() * workspace.element_size(), _stream()))
        return y
    fn = abi.lib().lotus_gemm_bias_fwd if force_gemm else abi.lib().lotus_linear_fwd
    check(fn(_ptr(x), _ptr(w_packed), _ptr(bias), _ptr(y), m, in_f, out_f, act,
             OUT_ROWS_F32 if out_f32 else OUT_NHWC_F16, _stream()))
    return y


def gemv(w: torch.Tensor, x: torch.Tensor, bias: Optional[torch.Tensor], act=ACT_NONE, w_in: Optional[int] = None,
         h_out: Optional[int] = None, y_f16=False) -> torch.Tensor:
    """Reference Fgemva semantics: y[b, h] = act(W[h,:] . x[b,:] + bias[h])."""
    w_f16 = 1 if w.dtype == torch.float16 else 0
    x_f16 = 1 if x.dtype == torch.float16 else 0
    h_out = h_out if h_out is not None else w.shape[0]
    w_in = w_in if w_in is not None else (w.shape[1] if not w_f16 else x.shape[-1])
    x2 = x if x.dim() == 2 else x.view(1, -1)
    batch = x2.shape[0]
    if y_f16:
        y = torch.empty((batch, channel_stride(h_out)), dtype=torch.float16, device=w.device)
    else:
        y = torch.empty((batch, h_out), dtype=torch.float32, device=w.device)
    check(abi.lib().lotus_gemv_bias_fwd(_ptr(w), w_f16, _ptr(x2), x_f16, _ptr(bias), _ptr(y), 1 if y_f16 else 0,
                                        batch, h_out, w_in, act, _stream()))
    return y


# --------------------------------------------------------------------- pooling / eltwise
def maxpool2d(x: torch.Tensor, c: int, k, stride, pad=0, act=ACT_NONE) -> torch.Tensor:
    n, h, w, cs = x.shape
    kh, kw = _pair(k)
    sh, sw = _pair(stride)
    ph, pw = _pair(pad)
    d = Pool2dDesc(n, c, h, w, kh, kw, sh, sw, ph, pw, act)
    oh, ow = ctypes.c_int(), ctypes.c_int()
    check(abi.lib().lotus_maxpool2d_out_hw(ctypes.byref(d), ctypes.byref(oh), ctypes.byref(ow)))
    y = torch.empty((n, oh.value, ow.value, cs), dtype=torch.float16, device=x.device)
    check(abi.lib().lotus_maxpool2d_fwd(_ptr(x), _ptr(y), ctypes.byref(d), _stream()))
    return y


def conv2d_maxpool(x: torch.Tensor, c_in: int, w_packed: torch.Tensor, bias: Optional[torch.Tensor], c_out: int,
                   k, act=ACT_NONE, pool: bool = True) -> torch.Tensor:
    """Row-tile conv (stride 1, no padding) with the fused 3x3/2 pad-1 max
    pool, or without the pool when pool=False; NHWC fp16 in and out."""
    n, h, w, _ = x.shape
    kh, kw = _pair(k)
    d = conv_desc(n, c_in, h, w, c_out, (kh, kw), 1, 0, act)
    oh, ow = h - kh + 1, w - kw + 1
    pd = Pool2dDesc(n, c_out, oh, ow, 3, 3, 2, 2, 1, 1, ACT_NONE) if pool else None
    if pool:
        oh, ow = (oh - 1) // 2 + 1, (ow - 1) // 2 + 1
    y = torch.empty((n, oh, ow, channel_stride(c_out)), dtype=torch.float16, device=x.device)
    check(abi.lib().lotus_conv2d_maxpool_fwd(_ptr(x), _ptr(w_packed), _ptr(bias), _ptr(y), ctypes.byref(d),
                                             ctypes.byref(pd) if pool else None, _stream()))
    return y


def adaptive_avgpool2d(x: torch.Tensor, c: int, out_hw, act=ACT_NONE, out_f32=False) -> torch.Tensor:
    n, h, w, cs = x.shape
    oh, ow = _pair(out_hw)
    if out_f32:
        y = torch.empty((n, oh * ow * c), dtype=torch.float32, device=x.device)
    else:
        y = torch.empty((n, oh, ow, cs), dtype=torch.float16, device=x.device)
    check(abi.lib().lotus_adaptive_avgpool2d_fwd(_ptr(x), _ptr(y), n, c, h, w, oh, ow, act, 1 if out_f32 else 0,
                                                 _stream()))
    return y


def add_act(a: torch.Tensor, b: torch.Tensor, c: int, act=ACT_NONE) -> torch.Tensor:
    assert a.shape == b.shape
    y = torch.empty_like(a)
    pixels = a.numel() // a.shape[-1]
    check(abi.lib().lotus_add_act_fwd(_ptr(a), _ptr(b), _ptr(y), pixels, c, act, _stream()))
    return y


def concat_channels(a: torch.Tensor, ca: int, b: torch.Tensor, cb: int) -> torch.Tensor:
    n, h, w, _ = a.shape
    y = torch.empty((n, h, w, channel_stride(ca + cb)), dtype=torch.float16, device=a.device)
    check(abi.lib().lotus_concat_channels_fwd(_ptr(a), ca, _ptr(b), cb, _ptr(y), n, h, w, _stream()))
    return y


# --------------------------------------------------------------------- input preprocessing
def preprocess_bgr_u8(images: torch.Tensor, resize_hw=(256, 256), crop_hw=(224, 224)) -> torch.Tensor:
    """[n, h, w, 3] uint8 BGR device images -> [n, 3, crop_h, crop_w] fp32
    (lotus_preprocess_bgr_u8 with the reference's ImageNet constants)."""
    n, h, w, _ = images.shape
    y = torch.empty((n, 3) + tuple(crop_hw), dtype=torch.float32, device=images.device)
    check(abi.lib().lotus_preprocess_bgr_u8(_ptr(images.contiguous()), n, h, w, resize_hw[0], resize_hw[1], crop_hw[0],
                                            crop_hw[1], None, None, _ptr(y), _stream()))
    return y
