"""The drop-in boundary exercised from compiled C++.

tests/cpp/dropin_caller.cpp is a reference-style caller: a Conv2dLayer whose
Forward takes and returns the reference's NCHW fp32 device tensors and wraps
lotus_conv2d_fwd with the NHWC fp16 layout conversions (the binding
INTEGRATION.md shows), and the Graph sequence InitialiseInput / Forward /
Output through lotus_graph_*.  The tests build it with tests/cpp/Makefile, run
it on seeded inputs and compare its outputs with the CPU oracle.
"""
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle
from tests._metrics import assert_close, max_abs, rel_l2

pytestmark = pytest.mark.gpu

CPP = os.path.join(os.path.dirname(os.path.abspath(__file__)), "cpp")
EXE = os.path.join(CPP, "dropin_caller")


@pytest.fixture(scope="module")
def exe():
    subprocess.run(["make", "-s", "-C", CPP], check=True)
    return EXE


@pytest.mark.parametrize("case", [
    # n, c, h, w, cout, k, stride, pad, act
    (1, 64, 56, 56, 64, 3, 1, 1, 1),    # the single-conv benchmark shape
    (2, 3, 40, 40, 17, 7, 2, 3, 0),     # a stem-like 7x7/2 with an odd channel count
    (2, 128, 14, 14, 256, 3, 2, 1, 2),  # strided, sigmoid
])
def test_cpp_conv2d_layer_nchw_f32(exe, tmp_path, case):
    n, c, h, w, cout, k, s, p, act = case
    rng = np.random.default_rng(sum(case))
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, np.sqrt(2.0 / (c * k * k)), (cout, c, k, k)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    inp, out = tmp_path / "in.bin", tmp_path / "out.bin"
    with open(inp, "wb") as f:
        f.write(np.array(case, np.int32).tobytes())
        f.write(x.tobytes())
        f.write(wt.tobytes())
        f.write(b.tobytes())
    subprocess.run([exe, "conv", str(inp), str(out)], check=True)
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    got = np.fromfile(out, np.float32).reshape(n, cout, oh, ow)
    assert_close(got, oracle.conv2d(x, wt, b, (s, s), (p, p), act), what=str(case))


def test_cpp_graph_forward(exe, tmp_path):
    from lotusinfer_b200 import synth
    param, binp = synth.make_model("resnet18", str(tmp_path), seed=0)
    x = synth.synthetic_input("resnet18", 3, seed=5)
    inp, out = tmp_path / "x.bin", tmp_path / "y.bin"
    x.tofile(inp)
    subprocess.run([exe, "graph", param, binp, "3", str(inp), str(out)], check=True)
    got = np.fromfile(out, np.float32).reshape(3, 1000)
    want = oracle.run_graph(param, binp, x)
    assert max_abs(got, want) <= 5e-3 * float(np.abs(want).max())
    assert rel_l2(got, want) <= 5e-3
    assert np.array_equal(np.argmax(got, 1), np.argmax(want, 1))
