"""Run one ResNet-18 convolution layer shape through the C ABI (profiling aid).

    python -m lotusinfer_b200.conv_probe --layer s1 --batch 256 --reps 3

Layers (ResNet-18 at batch B, NHWC fp16, seeded random data):
  stem  3->64   7x7/2 on 224x224     s1   64->64   3x3/1 on 56x56 (+residual)
  stem_s2d 12->64 4x4/1 on 115x115 (the stem after the graph's space-to-depth rewrite)
  s2d  64->128  3x3/2 on 56x56       s2  128->128  3x3/1 on 28x28
  s3  256->256  3x3/1 on 14x14       s4  512->512  3x3/1 on 7x7
  ds2  64->128  1x1/2 on 56x56
Prints the mean device time per launch (CUDA events) and TFLOP/s.  With
--reps R the layer is launched R times after one warm-up launch, so an ncu
capture can select a single launch with `-k regex:conv_tc -s 1 -c 1`.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import kernels as K

LAYERS = {
    "stem": (3, 224, 224, 64, 7, 2, 3, False),
    "stem_s2d": (12, 115, 115, 64, 4, 1, 0, False),
    "s1": (64, 56, 56, 64, 3, 1, 1, True),
    "s2d": (64, 56, 56, 128, 3, 2, 1, False),
    "s2": (128, 28, 28, 128, 3, 1, 1, True),
    "s3": (256, 14, 14, 256, 3, 1, 1, True),
    "s4": (512, 7, 7, 512, 3, 1, 1, True),
    "ds2": (64, 56, 56, 128, 1, 2, 0, False),
}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layer", default="s1", choices=sorted(LAYERS))
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args()
    c, h, w, cout, k, s, p, res = LAYERS[a.layer]
    torch.manual_seed(0)
    dev = torch.device("cuda:0")
    x = K.to_nhwc(torch.randn(a.batch, c, h, w, device=dev))
    wt = torch.randn(cout, c, k, k, device=dev) * (2.0 / (c * k * k)) ** 0.5
    wp = K.conv2d_prepack(wt, c)
    bias = torch.rand(cout, device=dev) * 0.2 - 0.1
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    r = K.to_nhwc(torch.randn(a.batch, cout, oh, ow, device=dev)) if res else None
    K.conv2d(x, c, wp, bias, cout, k, s, p, 1, residual=r)  # warm-up
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.reps):
        K.conv2d(x, c, wp, bias, cout, k, s, p, 1, residual=r)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.reps
    flops = 2.0 * a.batch * oh * ow * cout * c * k * k
    print(json.dumps({"layer": a.layer, "batch": a.batch, "ms": ms, "tflops": flops / ms / 1e9,
                      "gflop": flops / 1e9}))


if __name__ == "__main__":
    main()
