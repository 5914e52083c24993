"""Run whole-network forward passes through the native graph (profiling aid).

    python -m lotusinfer_b200.forward_probe --model resnet18 --batch 64 --passes 2

Builds the synthetic model, then runs `--passes` eager forward passes (no
CUDA-graph replay, so every layer is a separate launch an ncu capture can
select, e.g. `-k regex:conv_tc -s 20 -c 20` for the second ResNet-18 pass)
and prints the per-pass device time.
"""
from __future__ import annotations

import argparse
import json
import os
import tempfile

from . import synth
from .graph import Graph


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="resnet18", choices=sorted(synth.TOPOLOGIES))
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--passes", type=int, default=2)
    a = ap.parse_args()
    d = os.environ.get("LOTUS_MODEL_DIR", os.path.join(tempfile.gettempdir(), "lotus_models"))
    param, binp = synth.make_model(a.model, d, seed=0)
    g = Graph(param, binp, a.batch, cuda_graph=False)
    x = synth.synthetic_input(a.model, a.batch, seed=0)
    g.set_input(x)
    import torch
    s = torch.cuda.ExternalStream(g.stream)
    times = []
    for _ in range(a.passes):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        g.forward()
        e1.record(s)
        g.synchronize()
        times.append(e0.elapsed_time(e1))
    print(json.dumps({"model": a.model, "batch": a.batch, "pass_ms": times, "layers": len(g.layers())}))
    g.close()


if __name__ == "__main__":
    main()
