"""Synthetic PNNX models: topology writers and seeded random-weight archives.

The reference ships the three model topologies as .pnnx.param text but no
weights (its generators need torch.hub downloads).  This module writes the
same three topologies from their architecture descriptions and fills a
stored-zip .pnnx.bin with seeded random weights:

* ResNet-18: 7x7/2 stem + 3x3/2 maxpool, BasicBlocks [2,2,2,2] at widths
  64/128/256/512 with 1x1/2 downsample convs, BN folded into conv bias,
  residual add + ReLU, adaptive avgpool 1x1, flatten, FC 512->1000.
* U-Net (brain segmentation layout): 3 -> 32 features doubling to 512 over
  four 2x2-maxpool levels, two 3x3 conv+ReLU per block, 2x2/2 transposed-conv
  upsampling, channel concatenation skips, 1x1 conv + sigmoid.
* AlexNet: conv 11x11/4 64, 5x5 192, 3x3 384/256/256 with 3x3/2 maxpools,
  adaptive avgpool 6x6, FC 9216->4096->4096->1000 with ReLU.

Weights: Kaiming-normal (std = sqrt(2 / fan_in)) for conv, transposed conv
and linear weights, biases U(-0.1, 0.1).  File format: the .pnnx.param text
grammar and the stored-zip archive with "<op>.<attr>" entries of raw
little-endian fp32 that the reference loads (source/pnnx/ir.cpp:644-806).
"""
from __future__ import annotations

import os
import zipfile
from typing import Dict, List, Sequence, Tuple

import numpy as np

MAGIC = 7767517


def _fmt(v) -> str:
    if isinstance(v, bool):
        return "True" if v else "False"
    if isinstance(v, (tuple, list)):
        return "(" + ",".join(_fmt(e) for e in v) + ")"
    return str(v)


def _shape(s: Sequence[int]) -> str:
    return "(" + ",".join(str(int(d)) for d in s) + ")f32"


class ParamWriter:
    """Accumulates operators and operands and renders the .pnnx.param text."""

    def __init__(self):
        self.lines: List[str] = []
        self.shapes: Dict[str, Tuple[int, ...]] = {}
        self.n_operands = 0
        self.attrs: Dict[str, Tuple[int, ...]] = {}  # "<op>.<attr>" -> shape

    def _new(self, shape) -> str:
        name = str(self.n_operands)
        self.n_operands += 1
        self.shapes[name] = tuple(int(d) for d in shape)
        return name

    def op(self, type_: str, name: str, inputs: Sequence[str], out_shapes: Sequence[Sequence[int]],
           params: Dict[str, object] = None, attrs: Dict[str, Sequence[int]] = None, input_key: bool = False) -> List[str]:
        outs = [self._new(s) for s in out_shapes]
        toks = [f"{type_:<24}", f"{name:<24}", str(len(inputs)), str(len(outs))] + list(inputs) + outs
        for k, v in (params or {}).items():
            toks.append(f"{k}={_fmt(v)}")
        for k, s in (attrs or {}).items():
            toks.append(f"@{k}={_shape(s)}")
            self.attrs[f"{name}.{k}"] = tuple(s)
        if input_key and inputs:
            toks.append(f"$input={inputs[0]}")
        for o in list(inputs) + outs:
            toks.append(f"#{o}={_shape(self.shapes[o])}")
        self.lines.append(" ".join(toks))
        return outs

    def text(self) -> str:
        return f"{MAGIC}\n{len(self.lines)} {self.n_operands}\n" + "\n".join(self.lines) + "\n"

    # ---------------------------------------------------------------- helpers
    def input(self, shape) -> str:
        return self.op("pnnx.Input", "pnnx_input_0", [], [shape])[0]

    def output(self, x: str) -> None:
        toks = [f"{'pnnx.Output':<24}", f"{'pnnx_output_0':<24}", "1", "0", x, f"#{x}={_shape(self.shapes[x])}"]
        self.lines.append(" ".join(toks))

    def conv(self, name, x, cout, k, s=1, p=0, bias=True) -> str:
        n, cin, h, w = self.shapes[x]
        oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
        attrs = {"bias": (cout,), "weight": (cout, cin, k, k)} if bias else {"weight": (cout, cin, k, k)}
        return self.op("nn.Conv2d", name, [x], [(n, cout, oh, ow)],
                       {"bias": bias, "dilation": (1, 1), "groups": 1, "in_channels": cin, "kernel_size": (k, k),
                        "out_channels": cout, "padding": (p, p), "padding_mode": "zeros", "stride": (s, s)},
                       attrs, input_key=True)[0]

    def tconv(self, name, x, cout, k, s) -> str:
        n, cin, h, w = self.shapes[x]
        oh, ow = (h - 1) * s + k, (w - 1) * s + k
        return self.op("nn.ConvTranspose2d", name, [x], [(n, cout, oh, ow)],
                       {"bias": True, "dilation": (1, 1), "groups": 1, "in_channels": cin, "kernel_size": (k, k),
                        "out_channels": cout, "output_padding": (0, 0), "padding": (0, 0), "stride": (s, s)},
                       {"bias": (cout,), "weight": (cin, cout, k, k)})[0]

    def relu(self, name, x) -> str:
        return self.op("nn.ReLU", name, [x], [self.shapes[x]])[0]

    def sigmoid(self, name, x) -> str:
        return self.op("F.sigmoid", name, [x], [self.shapes[x]], input_key=True)[0]

    def maxpool(self, name, x, k, s, p=0) -> str:
        n, c, h, w = self.shapes[x]
        oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
        return self.op("nn.MaxPool2d", name, [x], [(n, c, oh, ow)],
                       {"ceil_mode": False, "dilation": (1, 1), "kernel_size": (k, k), "padding": (p, p),
                        "return_indices": False, "stride": (s, s)})[0]

    def add(self, name, a, b) -> str:
        return self.op("pnnx.Expression", name, [a, b], [self.shapes[a]], {"expr": "add(@0,@1)"})[0]

    def avgpool(self, name, x, out) -> str:
        n, c, _, _ = self.shapes[x]
        return self.op("nn.AdaptiveAvgPool2d", name, [x], [(n, c, out, out)], {"output_size": (out, out)})[0]

    def flatten(self, name, x) -> str:
        s = self.shapes[x]
        return self.op("torch.flatten", name, [x], [(s[0], int(np.prod(s[1:])))], {"end_dim": -1, "start_dim": 1},
                       input_key=True)[0]

    def linear(self, name, x, out_f) -> str:
        n, in_f = self.shapes[x]
        return self.op("nn.Linear", name, [x], [(n, out_f)],
                       {"bias": True, "in_features": in_f, "out_features": out_f},
                       {"bias": (out_f,), "weight": (out_f, in_f)})[0]

    def cat(self, name, a, b) -> str:
        n, ca, h, w = self.shapes[a]
        cb = self.shapes[b][1]
        return self.op("torch.cat", name, [a, b], [(n, ca + cb, h, w)], {"dim": 1})[0]


# ------------------------------------------------------------------ topologies
def resnet18() -> ParamWriter:
    g = ParamWriter()
    x = g.input((1, 3, 224, 224))
    ci = [0]

    def conv(x, cout, k, s, p):
        name = f"convbn2d_{ci[0]}"
        ci[0] += 1
        return g.conv(name, x, cout, k, s, p)

    x = g.relu("relu", conv(x, 64, 7, 2, 3))
    x = g.maxpool("maxpool", x, 3, 2, 1)
    expr = [14]
    uniq = [0]
    for stage, width in enumerate((64, 128, 256, 512), start=1):
        for blk in range(2):
            stride = 2 if (stage > 1 and blk == 0) else 1
            identity = x
            y = g.relu(f"layer{stage}.{blk}.relu", conv(x, width, 3, stride, 1))
            y = conv(y, width, 3, 1, 1)
            if stride != 1:
                identity = conv(x, width, 1, stride, 0)
            y = g.add(f"pnnx_expr_{expr[0]}", y, identity)
            expr[0] -= 2
            x = g.relu(f"pnnx_unique_{uniq[0]}", y)
            uniq[0] += 1
    x = g.avgpool("avgpool", x, 1)
    x = g.flatten("torch.flatten_0", x)
    x = g.linear("fc", x, 1000)
    g.output(x)
    return g


def unet() -> ParamWriter:
    g = ParamWriter()
    x = g.input((1, 3, 256, 256))
    ci = [0]

    def block(x, cout, tag):
        for j in (1, 2):
            name = f"convbn2d_{ci[0]}"
            ci[0] += 1
            x = g.relu(f"{tag}relu{j}", g.conv(name, x, cout, 3, 1, 1))
        return x

    skips = []
    feats = 32
    for lvl in range(1, 5):
        x = block(x, feats * 2 ** (lvl - 1), f"encoder{lvl}.enc{lvl}")
        skips.append(x)
        x = g.maxpool(f"pool{lvl}", x, 2, 2)
    x = block(x, feats * 16, "bottleneck.bottleneck")
    for lvl in range(4, 0, -1):
        x = g.tconv(f"upconv{lvl}", x, feats * 2 ** (lvl - 1), 2, 2)
        x = g.cat(f"torch.cat_{5 - lvl}", x, skips[lvl - 1])
        x = block(x, feats * 2 ** (lvl - 1), f"decoder{lvl}.dec{lvl}")
    x = g.conv("conv", x, 1, 1, 1, 0)
    x = g.sigmoid("F.sigmoid_0", x)
    g.output(x)
    return g


def alexnet() -> ParamWriter:
    g = ParamWriter()
    x = g.input((1, 3, 224, 224))
    x = g.relu("features.1", g.conv("features.0", x, 64, 11, 4, 2))
    x = g.maxpool("features.2", x, 3, 2)
    x = g.relu("features.4", g.conv("features.3", x, 192, 5, 1, 2))
    x = g.maxpool("features.5", x, 3, 2)
    x = g.relu("features.7", g.conv("features.6", x, 384, 3, 1, 1))
    x = g.relu("features.9", g.conv("features.8", x, 256, 3, 1, 1))
    x = g.relu("features.11", g.conv("features.10", x, 256, 3, 1, 1))
    x = g.maxpool("features.12", x, 3, 2)
    x = g.avgpool("avgpool", x, 6)
    x = g.flatten("torch.flatten_0", x)
    x = g.relu("classifier.2", g.linear("classifier.1", x, 4096))
    x = g.relu("classifier.5", g.linear("classifier.4", x, 4096))
    x = g.linear("classifier.6", x, 1000)
    g.output(x)
    return g


TOPOLOGIES = {"resnet18": resnet18, "unet": unet, "alexnet": alexnet}
INPUT_SHAPES = {"resnet18": (3, 224, 224), "unet": (3, 256, 256), "alexnet": (3, 224, 224)}


# ------------------------------------------------------------------ weights
def random_weights(g: ParamWriter, seed: int) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    out = {}
    for key, shape in g.attrs.items():
        if key.endswith(".bias"):
            out[key] = rng.uniform(-0.1, 0.1, shape).astype(np.float32)
        else:
            if len(shape) == 4 and ".weight" in key and key.split(".")[0].startswith("upconv"):
                fan_in = shape[0]  # transposed conv [Cin, Cout, k, k] with stride == kernel: Cin terms per output
            else:
                fan_in = int(np.prod(shape[1:]))
            out[key] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(np.sqrt(2.0 / fan_in)))
    return out


def write_bin(path: str, weights: Dict[str, np.ndarray]) -> None:
    """Stored (uncompressed) zip with one raw fp32 entry per attribute."""
    tmp = f"{path}.{os.getpid()}.tmp"  # concurrent writers (one per rank) never share a temporary
    with zipfile.ZipFile(tmp, "w", compression=zipfile.ZIP_STORED, allowZip64=True) as z:
        for key in sorted(weights):
            z.writestr(zipfile.ZipInfo(key), np.ascontiguousarray(weights[key], "<f4").tobytes())
    os.replace(tmp, path)


def make_model(name: str, out_dir: str, seed: int = 0) -> Tuple[str, str]:
    """Write <name>.pnnx.param and <name>_s<seed>.pnnx.bin under out_dir (cached)."""
    os.makedirs(out_dir, exist_ok=True)
    g = TOPOLOGIES[name]()
    param = os.path.join(out_dir, f"{name}.pnnx.param")
    binp = os.path.join(out_dir, f"{name}_s{seed}.pnnx.bin")
    text = g.text()
    if not os.path.exists(param) or open(param).read() != text:
        tmp = f"{param}.{os.getpid()}.tmp"
        with open(tmp, "w") as f:
            f.write(text)
        os.replace(tmp, param)
    if not os.path.exists(binp):
        write_bin(binp, random_weights(g, seed))
    return param, binp


def synthetic_input(name: str, batch: int, seed: int = 0) -> np.ndarray:
    """ResNet/AlexNet inputs ~N(0,1), U-Net inputs ~U(0,1), NCHW fp32."""
    rng = np.random.default_rng(1000 + seed)
    shape = (batch,) + INPUT_SHAPES[name]
    if name == "unet":
        return rng.uniform(0.0, 1.0, shape).astype(np.float32)
    return rng.standard_normal(shape, dtype=np.float32)
