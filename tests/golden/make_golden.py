"""Generate golden fixtures by running the reference's own operator kernels.

    make -C oracle/ref                      # needs the reference sources (build machine)
    python tests/golden/make_golden.py [out.npz]   # needs a CUDA GPU

The reference kernels (compiled from the reference tree into
oracle/_ref/libref_ops.so through oracle/ref/ref_launch.cu, which repeats the
reference layers' per-sample launch loops) run on seeded inputs; inputs and
outputs are saved to tests/golden/ref_ops.npz, against which
tests/test_golden_cpu.py checks the CPU oracle.  Inputs stay inside what each
reference kernel handles in bounds: maxpool without padding (its running max
starts uninitialised on padded windows), GEMM with m <= n, GEMV on its
element-wise path (width not a multiple of 4, height a multiple of 8).
Integer-valued inputs make the fp32 reference results exact, so those cases
pin the oracle bit for bit.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
LIB = os.path.join(ROOT, "oracle", "_ref", "libref_ops.so")

CONV = [  # name, n, c, h, w, cout, k, s, p, act, integer data
    ("conv_7x7s2_cin3_cout17", 2, 3, 31, 29, 17, 7, 2, 1, 0, True),
    ("conv_3x3_relu", 1, 16, 14, 14, 24, 3, 1, 1, 1, False),
    ("conv_5x5s3_sigmoid", 2, 8, 9, 11, 5, 5, 3, 2, 2, False),
    ("conv_1x1s2", 2, 32, 10, 10, 16, 1, 2, 0, 0, True),
]
TCONV = [  # name, n, cin, h, w, cout, k, s, act
    ("tconv_k2s3_gaps", 1, 16, 20, 20, 8, 2, 3, 0),
    ("tconv_k2s2_unet", 2, 32, 8, 8, 16, 2, 2, 1),
]
MAXPOOL = [("maxpool_3x3s2", 1, 3, 33, 33, 3, 2, 0), ("maxpool_2x2s2_relu", 2, 8, 16, 16, 2, 2, 1)]
AAP = [("aap_7to1", 2, 16, 7, 7, 1, 1), ("aap_refwin_33to8", 1, 3, 33, 33, 8, 8)]


def main(out_path: str) -> None:
    lib = ctypes.CDLL(LIB)
    P = ctypes.c_void_p
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(20261201)
    store = {}

    keep = []  # device tensors stay referenced until every launch has finished

    def g(a):
        t = torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)
        keep.append(t)
        return t

    def ptr(t):
        return P(t.data_ptr()) if t is not None else None

    for name, n, c, h, w, cout, k, s, p, act, integer in CONV:
        if integer:
            x = rng.integers(-5, 5, (n, c, h, w)).astype(np.float32)
            wt = rng.integers(-10, 10, (cout, c, k, k)).astype(np.float32)
            b = rng.integers(-10, 10, cout).astype(np.float32)
        else:
            x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
            wt = rng.normal(0, np.sqrt(2.0 / (c * k * k)), (cout, c, k, k)).astype(np.float32)
            b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
        oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
        y = torch.zeros((n, cout, oh, ow), dtype=torch.float32, device=dev)
        assert lib.ref_conv2d(ptr(g(x)), ptr(g(wt)), ptr(g(b)), ptr(y), n, c, h, w, cout, k, k, s, s, p, p, act) == 0
        store.update({f"{name}/x": x, f"{name}/w": wt, f"{name}/b": b, f"{name}/y": y.cpu().numpy(),
                      f"{name}/cfg": np.array([s, p, act], np.int32)})

    for name, n, cin, h, w, cout, k, s, act in TCONV:
        x = rng.integers(-10, 10, (n, cin, h, w)).astype(np.float32)
        wt = rng.integers(-10, 10, (cin, cout, k, k)).astype(np.float32)
        b = rng.integers(-10, 10, cout).astype(np.float32)
        oh, ow = (h - 1) * s + k, (w - 1) * s + k
        y = torch.zeros((n, cout, oh, ow), dtype=torch.float32, device=dev)
        assert lib.ref_tconv2d(ptr(g(x)), ptr(g(wt)), ptr(g(b)), ptr(y), n, cin, h, w, cout, k, k, s, s, act) == 0
        store.update({f"{name}/x": x, f"{name}/w": wt, f"{name}/b": b, f"{name}/y": y.cpu().numpy(),
                      f"{name}/cfg": np.array([s, act], np.int32)})

    for name, n, c, h, w, k, s, act in MAXPOOL:
        x = rng.normal(0, 1, (n, c, h, w)).astype(np.float32)
        oh, ow = (h - k) // s + 1, (w - k) // s + 1
        y = torch.zeros((n, c, oh, ow), dtype=torch.float32, device=dev)
        assert lib.ref_maxpool2d(ptr(g(x)), ptr(y), n, c, h, w, k, s, act) == 0
        store.update({f"{name}/x": x, f"{name}/y": y.cpu().numpy(), f"{name}/cfg": np.array([k, s, act], np.int32)})

    for name, n, c, h, w, oh, ow in AAP:
        x = rng.normal(0, 1, (n, c, h, w)).astype(np.float32)
        y = torch.zeros((n, c, oh, ow), dtype=torch.float32, device=dev)
        assert lib.ref_adaptive_avgpool2d(ptr(g(x)), ptr(y), n, c, h, w, oh, ow, 0) == 0
        store.update({f"{name}/x": x, f"{name}/y": y.cpu().numpy(), f"{name}/cfg": np.array([oh, ow], np.int32)})

    a = rng.normal(0, 1, 10000).astype(np.float32)
    b2 = rng.normal(0, 1, 10000).astype(np.float32)
    y = torch.zeros(10000, dtype=torch.float32, device=dev)
    assert lib.ref_add(ptr(g(a)), ptr(g(b2)), ptr(y), 10000, 1) == 0
    store.update({"add_relu/a": a, "add_relu/b": b2, "add_relu/y": y.cpu().numpy()})

    # GEMM (WMMA fp16 operands): fp16-representable inputs make every product exact
    m, n_, k = 40, 72, 100
    A = (rng.integers(-64, 64, (m, k)) / 16.0).astype(np.float32)
    B = (rng.integers(-64, 64, (n_, k)) / 16.0).astype(np.float32)
    bias = (rng.integers(-16, 16, n_) / 4.0).astype(np.float32)
    y = torch.zeros((m, n_), dtype=torch.float32, device=dev)
    assert lib.ref_gemm(ptr(g(A)), ptr(g(B)), ptr(g(bias)), ptr(y), m, n_, k, 0) == 0
    store.update({"gemm/a": A, "gemm/w": B, "gemm/b": bias, "gemm/y": y.cpu().numpy()})

    hh, ww = 64, 1001
    W = rng.normal(0, np.sqrt(1.0 / ww), (hh, ww)).astype(np.float32)
    xv = rng.uniform(-1, 1, ww).astype(np.float32)
    bv = rng.uniform(-0.1, 0.1, hh).astype(np.float32)
    y = torch.zeros(hh, dtype=torch.float32, device=dev)
    assert lib.ref_gemv(ptr(g(xv)), ptr(g(W)), ptr(g(bv)), ptr(y), hh, ww, 0) == 0
    store.update({"gemv/w": W, "gemv/x": xv, "gemv/b": bv, "gemv/y": y.cpu().numpy()})

    os.makedirs(os.path.dirname(os.path.abspath(out_path)), exist_ok=True)
    np.savez_compressed(out_path, **store)
    print(f"wrote {out_path}: {len(store)} arrays, {os.path.getsize(out_path)} bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(ROOT, "tests", "golden", "ref_ops.npz"))
