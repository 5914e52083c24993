"""Whole-network parity: the native graph runtime against the CPU oracle's
graph runner on the same synthetic PNNX model files.

Per-network tolerance: logits/masks within max-abs 5e-2 and rel-L2 5e-3 of the
fp32 oracle (activations are stored as fp16 between layers, so per-layer
rounding compounds over 18-23 layers); ResNet-18 / AlexNet top-1 identical on
every image whose oracle top-1/top-2 margin exceeds 10x the measured max-abs
error; U-Net masks (sigmoid > 0.5) identical outside the same band.
"""
import numpy as np
import pytest

from oracle import oracle
from tests._metrics import max_abs, rel_l2

pytestmark = pytest.mark.gpu

NET_MAX_ABS = 5e-2
NET_REL_L2 = 5e-3


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("models"))


def _graph(name, model_dir, batch, **kw):
    from lotusinfer_b200 import synth
    from lotusinfer_b200.graph import Graph
    param, binp = synth.make_model(name, model_dir, seed=0)
    return Graph(param, binp, batch, **kw), param, binp


def _top1_check(got, want):
    err = max_abs(got, want)
    srt = np.sort(want, axis=1)
    margin = srt[:, -1] - srt[:, -2]
    decisive = margin > 10 * err
    same = np.argmax(got, 1) == np.argmax(want, 1)
    assert np.all(same[decisive]), (margin, err)
    return int(decisive.sum()), int(same.sum())


@pytest.mark.parametrize("batch", [1, 4])
def test_resnet18_matches_oracle(model_dir, batch):
    from lotusinfer_b200 import synth
    g, param, binp = _graph("resnet18", model_dir, batch)
    x = synth.synthetic_input("resnet18", batch, seed=0)
    got = g.run(x)
    want = oracle.run_graph(param, binp, x)
    assert got.shape == want.shape == (batch, 1000)
    assert max_abs(got, want) <= NET_MAX_ABS * max(1.0, float(np.abs(want).max()) / 10)
    assert rel_l2(got, want) <= NET_REL_L2, rel_l2(got, want)
    _top1_check(got, want)
    g.close()


def test_resnet18_cuda_graph_replay_and_fusion_equivalence(model_dir):
    from lotusinfer_b200 import synth
    x = synth.synthetic_input("resnet18", 3, seed=1)
    g, _, _ = _graph("resnet18", model_dir, 3)
    first = g.run(x)            # eager
    second = g.run(x)           # captured + replayed
    third = g.run(x)            # replayed
    np.testing.assert_array_equal(first, second)
    np.testing.assert_array_equal(second, third)
    types = [l["type"] for l in g.layers()]
    assert "pnnx.Expression" not in types  # every residual add folded into a conv epilogue
    g.close()
    g2, _, _ = _graph("resnet18", model_dir, 3, fuse_residual=False, cuda_graph=False)
    assert "pnnx.Expression" in [l["type"] for l in g2.layers()]
    unfused = g2.run(x)
    # separate add kernel rounds the conv output to fp16 before the add: tiny differences only
    assert rel_l2(unfused, first) < 2e-3
    g2.close()


def test_unet_matches_oracle(model_dir):
    from lotusinfer_b200 import synth
    g, param, binp = _graph("unet", model_dir, 1)
    x = synth.synthetic_input("unet", 1, seed=0)
    got = g.run(x)
    want = oracle.run_graph(param, binp, x)
    assert got.shape == want.shape == (1, 1, 256, 256)
    err = max_abs(got, want)
    assert err <= NET_MAX_ABS and rel_l2(got, want) <= NET_REL_L2, (err, rel_l2(got, want))
    band = np.abs(want - 0.5) <= 10 * err
    assert np.array_equal((got > 0.5)[~band], (want > 0.5)[~band])
    g.close()


@pytest.mark.parametrize("batch", [2, 12])
def test_alexnet_matches_oracle(model_dir, batch):
    """batch 2 runs the FC layers on the GEMV path, batch 12 on the tcgen05 GEMM."""
    from lotusinfer_b200 import synth
    g, param, binp = _graph("alexnet", model_dir, batch)
    x = synth.synthetic_input("alexnet", batch, seed=0)
    got = g.run(x)
    want = oracle.run_graph(param, binp, x)
    assert got.shape == want.shape == (batch, 1000)
    assert rel_l2(got, want) <= NET_REL_L2, rel_l2(got, want)
    _top1_check(got, want)
    g.close()


S2D_STEM = {"resnet18": 2, "alexnet": 4}  # stem stride = space-to-depth factor


def _s2d_weight(w, f):
    """W'[co, (a*f+b)*C + c, r', s'] = W[co, c, f*r' + a, f*s' + b] (zero past the kernel)."""
    co, c, kh, kw = w.shape
    kh2, kw2 = -(-kh // f), -(-kw // f)
    out = np.zeros((co, c * f * f, kh2, kw2), np.float32)
    for r in range(kh):
        for q in range(kw):
            a, b = r % f, q % f
            out[:, (a * f + b) * c:(a * f + b + 1) * c, r // f, q // f] = w[:, :, r, q]
    return out


def test_s2d_stem_matches_direct_stem(model_dir):
    """The space-to-depth stem rewrite leaves ResNet-18 and AlexNet outputs unchanged up to fp16 rounding."""
    from lotusinfer_b200 import synth
    for name in ("resnet18", "alexnet"):
        x = synth.synthetic_input(name, 2, seed=3)
        g1, _, _ = _graph(name, model_dir, 2)
        g2, _, _ = _graph(name, model_dir, 2, s2d_stem=False)
        a, b = g1.run(x), g2.run(x)
        assert rel_l2(a, b) < 2e-3, (name, rel_l2(a, b))
        g1.close()
        g2.close()


@pytest.mark.parametrize("name", ["resnet18", "unet", "alexnet"])
def test_graph_packed_weights_equal_standalone_prepack(model_dir, name):
    """Every layer's packed weights inside the runtime equal the standalone
    prepack of the same archive entry (guards the upload -> prepack ordering)."""
    import torch
    from lotusinfer_b200 import kernels as K
    from oracle import pnnx_text
    g, param, binp = _graph(name, model_dir, 1)
    pg = pnnx_text.load(param)
    W = pnnx_text.shaped_weights(pg, pnnx_text.read_weights(binp))
    chw = {}
    if name == "alexnet":
        chw["classifier.1"] = (256, 6, 6)
    for i, layer in enumerate(g.layers()):
        w = g.layer_weight(i)
        if w is None:
            continue
        n = layer["name"]
        w_np = W[n + ".weight"]
        if i == 1 and layer["type"] == "nn.Conv2d" and name in S2D_STEM:
            w_np = _s2d_weight(w_np, S2D_STEM[name])  # the stem runs over the space-to-depth input
        wt = torch.from_numpy(w_np).cuda()
        if layer["type"] == "nn.ConvTranspose2d":
            ref = K.tconv2d_prepack(wt)
        elif layer["type"] == "nn.Linear":
            ref = K.linear_prepack(wt, chw.get(n))
        else:
            ref = K.conv2d_prepack(wt, wt.shape[1])
        ref = ref.cpu().numpy().ravel()
        assert np.array_equal(w.view(np.uint16), ref.view(np.uint16)), n
    g.close()
