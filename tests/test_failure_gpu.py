"""Failure detection on the GPU without a GPU fault.

Every mbarrier wait in the conv kernel is bounded; a wait that runs out
records an error code in the device error word, the CTA drains its own
copies, frees its TMEM and returns.  These tests make such a wait run out on
purpose through the test hook LOTUS_TEST_WITHHOLD_ARRIVAL=1 (CTA 0's producer
skips its first load, so nothing ever completes that barrier phase) with a
short limit (LOTUS_WAIT_LIMIT try_wait rounds), then check that
  * lotus_device_error() reports the code and clears it,
  * the graph runtime turns it into a failed call instead of a success,
  * the context stays usable: the next normal launch passes parity.
No trap, no bad address and no unbounded wait is involved.
"""
import zlib

import numpy as np
import pytest

from oracle import oracle
from tests._metrics import assert_close

pytestmark = pytest.mark.gpu

WAIT_LIMIT = "2000"


def _cfg1(seed):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (1, 64, 56, 56)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / 576), (64, 64, 3, 3)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, 64).astype(np.float32)
    return x, w, b


def _run_conv(x, w, b):
    import torch
    from lotusinfer_b200 import kernels as K
    dev = torch.device("cuda:0")
    xg = K.to_nhwc(torch.from_numpy(x).to(dev))
    wp = K.conv2d_prepack(torch.from_numpy(w).to(dev), x.shape[1])
    y = K.conv2d(xg, x.shape[1], wp, torch.from_numpy(b).to(dev), w.shape[0], 3, 1, 1, 1)
    return K.from_nhwc(y, w.shape[0]).cpu().numpy()


@pytest.mark.parametrize("amode", ["", "1"])  # default (resident-weight halo) and the im2col pipeline
def test_expired_wait_is_reported_and_the_next_launch_is_correct(monkeypatch, amode):
    from lotusinfer_b200 import abi
    assert abi.device_error() == 0
    x, w, b = _cfg1(zlib.crc32(amode.encode()))
    if amode:
        monkeypatch.setenv("LOTUS_CONV_AMODE", amode)
    monkeypatch.setenv("LOTUS_WAIT_LIMIT", WAIT_LIMIT)
    monkeypatch.setenv("LOTUS_TEST_WITHHOLD_ARRIVAL", "1")
    _run_conv(x, w, b)
    code = abi.device_error()
    assert code in (1, 2, 3), code  # full / empty / accumulator wait expired
    assert abi.device_error() == 0  # read clears it
    monkeypatch.delenv("LOTUS_TEST_WITHHOLD_ARRIVAL")
    monkeypatch.delenv("LOTUS_WAIT_LIMIT")
    got = _run_conv(x, w, b)
    assert_close(got, oracle.conv2d(x, w, b, (1, 1), (1, 1), 1), what="after an expired wait")
    assert abi.device_error() == 0


def test_graph_call_fails_when_a_wait_expires(monkeypatch, tmp_path):
    from lotusinfer_b200 import abi, synth
    from lotusinfer_b200.abi import LotusError
    from lotusinfer_b200.graph import Graph
    param, binp = synth.make_model("resnet18", str(tmp_path), seed=0)
    x = synth.synthetic_input("resnet18", 1, seed=0)
    g = Graph(param, binp, 1, cuda_graph=False)  # eager: every launch reads the hook
    monkeypatch.setenv("LOTUS_WAIT_LIMIT", WAIT_LIMIT)
    monkeypatch.setenv("LOTUS_TEST_WITHHOLD_ARRIVAL", "1")
    g.set_input(x)
    with pytest.raises(LotusError, match="bounded wait expired"):
        g.forward_sync()
    monkeypatch.delenv("LOTUS_TEST_WITHHOLD_ARRIVAL")
    monkeypatch.delenv("LOTUS_WAIT_LIMIT")
    assert abi.device_error() == 0  # the failed call consumed the error word
    got = g.run(x)
    want = oracle.run_graph(param, binp, x)
    assert int(np.argmax(got)) == int(np.argmax(want))
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 5e-3
    g.close()
