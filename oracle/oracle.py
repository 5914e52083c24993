"""CPU oracle for the lotusInfer dense-contraction hot path (test infrastructure).

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` import this module, and only as the checker.  It wraps the C
restatements in ``oracle/lotus_oracle.c`` (fp32 NCHW, OpenMP) and adds a
whole-network runner for PNNX graphs (``run_graph``) that executes the
operators in the reference's graph order (source/graph.cpp:84-109, Kahn order
of source/graph.cpp:5-40) with the fusion rules of the reference layers
(ReLU / sigmoid folded into the producing conv or linear,
source/layer/layer_conv2d.cu:129-141).

Pinned: tests/test_golden_cpu.py checks these functions against outputs of
the reference's own kernels (tests/golden/ref_ops.npz, see lotus_oracle.c).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Dict, Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liblotus_oracle.so")
_lib = None

_F = ctypes.POINTER(ctypes.c_float)


def build() -> str:
    """Compile oracle/lotus_oracle.c into oracle/liblotus_oracle.so."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        i = ctypes.c_int
        L.oracle_conv2d.argtypes = [_F, _F, _F, _F, _F] + [i] * 12
        L.oracle_tconv2d.argtypes = [_F, _F, _F, _F] + [i] * 14
        L.oracle_gemv.argtypes = [_F, _F, _F, _F, i, i, i, i]
        L.oracle_gemm.argtypes = [_F, _F, _F, _F, i, i, i, i]
        L.oracle_maxpool2d.argtypes = [_F, _F] + [i] * 12
        L.oracle_adaptive_avgpool2d.argtypes = [_F, _F] + [i] * 7
        L.oracle_avgpool_reference_windows.argtypes = [_F, _F] + [i] * 5
        L.oracle_add.argtypes = [_F, _F, _F, ctypes.c_long, i]
        L.oracle_concat.argtypes = [_F, i, _F, i, _F, i, ctypes.c_long]
        L.oracle_num_threads.restype = i
        L.oracle_set_threads.argtypes = [i]
        _lib = L
    return _lib


def _p(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_F)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def conv2d(x, w, b=None, stride=(1, 1), pad=(0, 0), act=0, residual=None) -> np.ndarray:
    """NCHW fp32 conv2d + bias (+ residual) + act."""
    x, w, b, residual = _f32(x), _f32(w), _f32(b), _f32(residual)
    n, c, h, wd = x.shape
    cout, cin, kh, kw = w.shape
    assert cin == c
    oh = (h + 2 * pad[0] - kh) // stride[0] + 1
    ow = (wd + 2 * pad[1] - kw) // stride[1] + 1
    y = np.empty((n, cout, oh, ow), np.float32)
    if residual is not None:
        assert residual.shape == y.shape
    lib().oracle_conv2d(_p(x), _p(w), _p(b), _p(residual), _p(y), n, c, h, wd, cout, kh, kw, stride[0], stride[1],
                        pad[0], pad[1], act)
    return y


def tconv2d(x, w, b=None, stride=(2, 2), pad=(0, 0), out_pad=(0, 0), act=0) -> np.ndarray:
    """NCHW fp32 ConvTranspose2d; w is [Cin, Cout, kh, kw]."""
    x, w, b = _f32(x), _f32(w), _f32(b)
    n, cin, h, wd = x.shape
    cin2, cout, kh, kw = w.shape
    assert cin2 == cin
    oh = (h - 1) * stride[0] - 2 * pad[0] + kh + out_pad[0]
    ow = (wd - 1) * stride[1] - 2 * pad[1] + kw + out_pad[1]
    y = np.empty((n, cout, oh, ow), np.float32)
    lib().oracle_tconv2d(_p(x), _p(w), _p(b), _p(y), n, cin, h, wd, cout, kh, kw, stride[0], stride[1], pad[0], pad[1],
                         out_pad[0], out_pad[1], act)
    return y


def gemv(wmat, x, b=None, act=0) -> np.ndarray:
    """y[batch, H] for W [H, Wd] and x [batch, Wd] (or [Wd])."""
    wmat, b = _f32(wmat), _f32(b)
    x = _f32(np.atleast_2d(x))
    hout, win = wmat.shape
    y = np.empty((x.shape[0], hout), np.float32)
    lib().oracle_gemv(_p(wmat), _p(x), _p(b), _p(y), x.shape[0], hout, win, act)
    return y


def gemm(a, bmat, bias=None, act=0) -> np.ndarray:
    """C = act(A @ B^T + bias); A [M,K], B [N,K]."""
    a, bmat, bias = _f32(a), _f32(bmat), _f32(bias)
    m, k = a.shape
    nn = bmat.shape[0]
    c = np.empty((m, nn), np.float32)
    lib().oracle_gemm(_p(a), _p(bmat), _p(bias), _p(c), m, nn, k, act)
    return c


def maxpool2d(x, kernel, stride, pad=(0, 0), act=0, zero_pad=False) -> np.ndarray:
    x = _f32(x)
    n, c, h, wd = x.shape
    oh = (h + 2 * pad[0] - kernel[0]) // stride[0] + 1
    ow = (wd + 2 * pad[1] - kernel[1]) // stride[1] + 1
    y = np.empty((n, c, oh, ow), np.float32)
    lib().oracle_maxpool2d(_p(x), _p(y), n, c, h, wd, kernel[0], kernel[1], stride[0], stride[1], pad[0], pad[1], act,
                           1 if zero_pad else 0)
    return y


def adaptive_avgpool2d(x, out_hw, act=0) -> np.ndarray:
    x = _f32(x)
    n, c, h, wd = x.shape
    y = np.empty((n, c, out_hw[0], out_hw[1]), np.float32)
    lib().oracle_adaptive_avgpool2d(_p(x), _p(y), n, c, h, wd, out_hw[0], out_hw[1], act)
    return y


def avgpool_reference_windows(x, out_hw) -> np.ndarray:
    """The reference's fixed-window formula (single image [C, H, W])."""
    x = _f32(x)
    c, h, wd = x.shape
    y = np.empty((c, out_hw[0], out_hw[1]), np.float32)
    lib().oracle_avgpool_reference_windows(_p(x), _p(y), c, h, wd, out_hw[0], out_hw[1])
    return y


def add(x1, x2, act=0) -> np.ndarray:
    x1, x2 = _f32(x1), _f32(x2)
    assert x1.shape == x2.shape
    y = np.empty_like(x1)
    lib().oracle_add(_p(x1), _p(x2), _p(y), x1.size, act)
    return y


def concat(a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    n, ca, h, wd = a.shape
    cb = b.shape[1]
    y = np.empty((n, ca + cb, h, wd), np.float32)
    lib().oracle_concat(_p(a), ca, _p(b), cb, _p(y), n, h * wd)
    return y


# --------------------------------------------------------------------- graphs
from . import pnnx_text  # noqa: E402  (independent PNNX reader for the oracle)


def run_graph(param_path: str, bin_path: str, x: np.ndarray, weights: Optional[Dict[str, np.ndarray]] = None
              ) -> np.ndarray:
    """Run a PNNX graph on the CPU oracle; x is the NCHW fp32 input batch."""
    g = pnnx_text.load(param_path)
    if weights is None:
        weights = pnnx_text.shaped_weights(g, pnnx_text.read_weights(bin_path))
    vals: Dict[str, np.ndarray] = {}
    consumers: Dict[str, list] = {}
    for op in g.ops:
        for i in op.inputs:
            consumers.setdefault(i, []).append(op)

    def act_after(op):
        outs = consumers.get(op.outputs[0], [])
        if len(outs) == 1 and outs[0].type in ("nn.ReLU", "F.sigmoid"):
            return (1 if outs[0].type == "nn.ReLU" else 2), outs[0].outputs[0]
        return 0, op.outputs[0]

    for op in g.ops:
        t = op.type
        if t == "pnnx.Input":
            vals[op.outputs[0]] = np.ascontiguousarray(x, dtype=np.float32)
        elif t == "pnnx.Output":
            return vals[op.inputs[0]]
        elif t in ("nn.ReLU", "F.sigmoid"):
            src = op.inputs[0]
            if op.outputs[0] not in vals:  # not folded into its producer
                a = 1 if t == "nn.ReLU" else 2
                v = vals[src]
                vals[op.outputs[0]] = add(v, np.zeros_like(v), a)
        elif t == "nn.Conv2d":
            p = op.params
            act, out = act_after(op)
            vals[out] = conv2d(vals[op.inputs[0]], weights[op.name + ".weight"],
                               weights.get(op.name + ".bias") if p.get("bias", True) else None,
                               tuple(p["stride"]), tuple(p["padding"]), act)
        elif t == "nn.ConvTranspose2d":
            p = op.params
            act, out = act_after(op)
            vals[out] = tconv2d(vals[op.inputs[0]], weights[op.name + ".weight"],
                                weights.get(op.name + ".bias") if p.get("bias", True) else None,
                                tuple(p["stride"]), tuple(p["padding"]), tuple(p.get("output_padding", (0, 0))), act)
        elif t == "nn.Linear":
            p = op.params
            act, out = act_after(op)
            xin = vals[op.inputs[0]]
            vals[out] = gemm(xin.reshape(xin.shape[0], -1), weights[op.name + ".weight"],
                             weights.get(op.name + ".bias") if p.get("bias", True) else None, act)
        elif t == "nn.MaxPool2d":
            p = op.params
            act, out = act_after(op)
            vals[out] = maxpool2d(vals[op.inputs[0]], tuple(p["kernel_size"]), tuple(p["stride"]),
                                  tuple(p["padding"]), act)
        elif t == "nn.AdaptiveAvgPool2d":
            act, out = act_after(op)
            vals[out] = adaptive_avgpool2d(vals[op.inputs[0]], tuple(op.params["output_size"]), act)
        elif t == "pnnx.Expression":
            expr = op.params["expr"]
            if not expr.startswith("add("):
                raise NotImplementedError(expr)
            act, out = act_after(op)
            vals[out] = add(vals[op.inputs[0]], vals[op.inputs[1]], act)
        elif t == "torch.flatten":
            v = vals[op.inputs[0]]
            vals[op.outputs[0]] = v.reshape(v.shape[0], -1)
        elif t == "torch.cat":
            vals[op.outputs[0]] = concat(vals[op.inputs[0]], vals[op.inputs[1]])
        else:
            raise NotImplementedError(t)
    raise RuntimeError("graph has no pnnx.Output")


IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def preprocess_bgr_u8(images, resize_hw=(256, 256), crop_hw=(224, 224), mean=IMAGENET_MEAN, std=IMAGENET_STD):
    """Input preprocessing of the reference's classification demo
    (demo/image_classification.cpp:9-44): 8-bit BGR HWC images [n, h, w, 3]
    -> bilinear resize (cv::resize INTER_LINEAR geometry: half-pixel centres,
    source index clamped to the edge) -> RGB -> /255 -> centre crop ->
    (x - mean) / std, planar [n, 3, crop_h, crop_w] fp32.  Computed in float32
    with every operation rounded on its own (no fused multiply-add), in the
    order the GPU kernel uses; OpenCV's 8-bit path rounds the resized value to
    uint8 with 11-bit fixed-point weights, which this float restatement does
    not (it stays within one 8-bit step of it)."""
    imgs = np.asarray(images)
    if imgs.ndim == 3:
        imgs = imgs[None]
    n, h, w, _ = imgs.shape
    rh, rw = resize_hw
    ch, cw = crop_hw
    y0, x0 = max(0, rh // 2 - ch // 2), max(0, rw // 2 - cw // 2)
    f32 = np.float32

    def axis(n_src, n_dst, first, count):
        scale = f32(n_src) / f32(n_dst)
        d = np.arange(first, first + count, dtype=np.float32)
        f = (d + f32(0.5)) * scale - f32(0.5)
        s = np.floor(f)
        a = (f - s).astype(np.float32)
        i0 = s.astype(np.int64)
        lo = i0 < 0
        a[lo] = 0
        i0[lo] = 0
        hi = i0 >= n_src - 1
        a[hi] = 0
        i0[hi] = n_src - 1
        i1 = np.minimum(i0 + 1, n_src - 1)
        return i0, i1, a

    yi0, yi1, ay = axis(h, rh, y0, ch)
    xi0, xi1, ax = axis(w, rw, x0, cw)
    out = np.empty((n, 3, ch, cw), np.float32)
    one = f32(1.0)
    inv255 = f32(1.0 / 255.0)
    for c in range(3):
        src = imgs[..., 2 - c].astype(np.float32)  # BGR -> RGB
        p00 = src[:, yi0][:, :, xi0]
        p01 = src[:, yi0][:, :, xi1]
        p10 = src[:, yi1][:, :, xi0]
        p11 = src[:, yi1][:, :, xi1]
        axr, ayr = ax[None, None, :], ay[None, :, None]
        top = (one - axr) * p00 + axr * p01
        bot = (one - axr) * p10 + axr * p11
        v = ((one - ayr) * top + ayr * bot) * inv255
        out[:, c] = (v - f32(mean[c])) / f32(std[c])
    return out
