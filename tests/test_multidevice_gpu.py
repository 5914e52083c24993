"""Two GPUs in one process: kernel launch attributes and SM counts are kept
per device (and per CUDA context), so convs and whole graphs run correctly on
device 1 after device 0 in the same process.  No peer memory is involved.
Skipped unless at least two GPUs are visible."""
import numpy as np
import pytest

from oracle import oracle
from tests._metrics import assert_close, rel_l2

pytestmark = pytest.mark.gpu


def _two_gpus():
    import torch
    return torch.cuda.is_available() and torch.cuda.device_count() >= 2


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_conv_on_two_devices_in_one_process():
    import torch
    from lotusinfer_b200 import abi
    from lotusinfer_b200 import kernels as K
    rng = np.random.default_rng(21)
    x = rng.uniform(-1, 1, (2, 64, 56, 56)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2.0 / 576), (64, 64, 3, 3)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, 64).astype(np.float32)
    want = oracle.conv2d(x, w, b, (1, 1), (1, 1), 1)
    xs_np = np.ascontiguousarray(x[:, :16, :30, :30])
    ws_np = rng.normal(0, np.sqrt(2.0 / 256), (64, 16, 4, 4)).astype(np.float32)
    want_s = oracle.maxpool2d(oracle.conv2d(xs_np, ws_np, b, (1, 1), (0, 0), 1), (3, 3), (2, 2), (1, 1))
    for dev in (0, 1, 0, 1):
        with torch.cuda.device(dev):
            d = torch.device("cuda", dev)
            xg = K.to_nhwc(torch.from_numpy(x).to(d))
            wp = K.conv2d_prepack(torch.from_numpy(w).to(d), 64)
            y = K.conv2d(xg, 64, wp, torch.from_numpy(b).to(d), 64, 3, 1, 1, 1)
            assert_close(K.from_nhwc(y, 64).cpu().numpy(), want, what=f"device {dev}")
            # the fused stem kernel (its own launch attribute) on each device too
            xs = K.to_nhwc(torch.from_numpy(xs_np).to(d))
            ys = K.conv2d_maxpool(xs, 16, K.conv2d_prepack(torch.from_numpy(ws_np).to(d), 16),
                                  torch.from_numpy(b).to(d), 64, 4, 1)
            assert_close(K.from_nhwc(ys, 64).cpu().numpy(), want_s, what=f"stem kernel, device {dev}")
    assert abi.device_error() == 0


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_graphs_on_two_devices_in_one_process(tmp_path):
    from lotusinfer_b200 import synth
    from lotusinfer_b200.graph import Graph
    param, binp = synth.make_model("resnet18", str(tmp_path), seed=0)
    x = synth.synthetic_input("resnet18", 2, seed=4)
    want = oracle.run_graph(param, binp, x)
    g0 = Graph(param, binp, 2, device=0)
    g1 = Graph(param, binp, 2, device=1)
    for g in (g0, g1, g0, g1):
        got = g.run(x)
        assert rel_l2(got, want) < 5e-3
        assert np.array_equal(np.argmax(got, 1), np.argmax(want, 1))
    g0.close()
    g1.close()
