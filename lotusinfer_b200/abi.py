"""ctypes binding of liblotus_b200.so (the C ABI in include/lotus_ops.h).

Every call goes through the exported ``extern "C"`` entry points with raw
device pointers; PyTorch is used only to own device memory and streams.  The
library must be present: there is no Python or CPU fallback, and importing a
compute function without the built library raises.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblotus_b200.so")

ACT_NONE, ACT_RELU, ACT_SIGMOID = 0, 1, 2
OUT_NHWC_F16, OUT_ROWS_F32 = 0, 1


class LotusError(RuntimeError):
    """A lotus_* entry point returned a negative status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"lotus status {status}: {message}")
        self.status = status


class Conv2dDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("n", "c_in", "h", "w", "c_out", "kh", "kw", "stride_h", "stride_w",
                                             "pad_h", "pad_w", "act", "out_kind")]


class TConv2dDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("n", "c_in", "h", "w", "c_out", "kh", "kw", "stride_h", "stride_w",
                                             "pad_h", "pad_w", "out_pad_h", "out_pad_w", "act")]


class Pool2dDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("n", "c", "h", "w", "kh", "kw", "stride_h", "stride_w", "pad_h", "pad_w",
                                             "act")]


# name -> (restype, argtypes)
_V, _I, _S, _U64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_uint64
_CD = ctypes.POINTER(Conv2dDesc)
_TD = ctypes.POINTER(TConv2dDesc)
_PD = ctypes.POINTER(Pool2dDesc)
_IP = ctypes.POINTER(ctypes.c_int)

SIGNATURES = {
    "lotus_conv2d_out_hw": (_I, [_CD, _IP, _IP]),
    "lotus_channel_stride": (_I, [_I]),
    "lotus_conv2d_packed_weight_bytes": (_S, [_CD]),
    "lotus_conv2d_prepack": (_I, [_V, _V, _CD, _V]),
    "lotus_conv2d_fwd": (_I, [_V, _V, _V, _V, _V, _CD, _V]),
    "lotus_conv2d_workspace_bytes": (_S, [_CD]),
    "lotus_conv2d_workspace_bytes_max": (_S, [_CD]),
    "lotus_conv2d_fwd_ws": (_I, [_V, _V, _V, _V, _V, _CD, _V, _S, _V]),
    "lotus_conv2d_fwd_noalloc": (_I, [_V, _V, _V, _V, _V, _CD, _V]),
    "lotus_conv2d_fwd_slice": (_I, [_V, _V, _V, _V, _V, _I, _CD, _V, _S, _V]),
    "lotus_tconv2d_out_hw": (_I, [_TD, _IP, _IP]),
    "lotus_tconv2d_packed_weight_bytes": (_S, [_TD]),
    "lotus_tconv2d_prepack": (_I, [_V, _V, _TD, _V]),
    "lotus_tconv2d_fwd": (_I, [_V, _V, _V, _V, _TD, _V]),
    "lotus_tconv2d_fwd_slice": (_I, [_V, _V, _V, _V, _I, _TD, _V]),
    "lotus_linear_packed_weight_bytes": (_S, [_I, _I]),
    "lotus_linear_prepack": (_I, [_V, _V, _I, _I, _I, _I, _I, _V]),
    "lotus_linear_fwd": (_I, [_V, _V, _V, _V, _I, _I, _I, _I, _I, _V]),
    "lotus_linear_workspace_bytes": (_S, [_I, _I, _I]),
    "lotus_linear_fwd_ws": (_I, [_V, _V, _V, _V, _I, _I, _I, _I, _I, _V, _S, _V]),
    "lotus_gemm_bias_fwd": (_I, [_V, _V, _V, _V, _I, _I, _I, _I, _I, _V]),
    "lotus_gemv_bias_fwd": (_I, [_V, _I, _V, _I, _V, _V, _I, _I, _I, _I, _I, _V]),
    "lotus_maxpool2d_out_hw": (_I, [_PD, _IP, _IP]),
    "lotus_maxpool2d_fwd": (_I, [_V, _V, _PD, _V]),
    "lotus_maxpool2d_fwd_strided": (_I, [_V, _I, _V, _PD, _V]),
    "lotus_conv2d_maxpool_supported": (_I, [_CD, _PD]),
    "lotus_conv2d_maxpool_fwd": (_I, [_V, _V, _V, _V, _CD, _PD, _V]),
    "lotus_adaptive_avgpool2d_fwd": (_I, [_V, _V, _I, _I, _I, _I, _I, _I, _I, _I, _V]),
    "lotus_add_act_fwd": (_I, [_V, _V, _V, _S, _I, _I, _V]),
    "lotus_concat_channels_fwd": (_I, [_V, _I, _V, _I, _V, _I, _I, _I, _V]),
    "lotus_nchw_f32_to_nhwc_f16": (_I, [_V, _V, _I, _I, _I, _I, _V]),
    "lotus_nhwc_f16_to_nchw_f32": (_I, [_V, _V, _I, _I, _I, _I, _V]),
    "lotus_space_to_depth_f16": (_I, [_V, _V, _I, _I, _I, _I, _I, _I, _I, _I, _I, _V]),
    "lotus_preprocess_bgr_u8": (_I, [_V, _I, _I, _I, _I, _I, _I, _I, _V, _V, _V, _V]),
    "lotus_last_error_string": (ctypes.c_char_p, []),
    "lotus_device_error": (_I, []),
    "lotus_launch_count": (_U64, []),
}

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Load liblotus_b200.so (built by lotusinfer_b200.build); raises if absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m lotusinfer_b200.build` (no fallback exists)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != 0:
        msg = lib().lotus_last_error_string()
        raise LotusError(status, msg.decode() if msg else "")


def last_error() -> str:
    return lib().lotus_last_error_string().decode()


def channel_stride(c: int) -> int:
    return (c + 7) // 8 * 8


def launch_count() -> int:
    return int(lib().lotus_launch_count())


def device_error() -> int:
    return int(lib().lotus_device_error())
