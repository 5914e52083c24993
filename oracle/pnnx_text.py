"""Independent PNNX reader for the CPU oracle (test infrastructure only).

Parses the ``.pnnx.param`` text format the reference loads in
source/pnnx/ir.cpp:700-806 (magic line, ``op_count operand_count``, then one
operator per line: type, name, input/output counts and operand names, then
``key=value`` items where ``@`` marks an attribute, ``#`` an operand shape and
``$`` an input key) and the stored-zip ``.pnnx.bin`` whose entries are named
``<op>.<attribute>`` (source/pnnx/ir.cpp:681) and hold raw little-endian data.
Parameter values follow Parameter::parse_from_string (source/pnnx/ir.cpp:327-406).
"""
from __future__ import annotations

import zipfile
from dataclasses import dataclass, field
from typing import Dict, List

import numpy as np


@dataclass
class Op:
    type: str
    name: str
    inputs: List[str]
    outputs: List[str]
    params: Dict[str, object] = field(default_factory=dict)
    attrs: Dict[str, tuple] = field(default_factory=dict)      # name -> (shape, type)
    shapes: Dict[str, tuple] = field(default_factory=dict)     # operand -> (shape, type)


@dataclass
class Graph:
    ops: List[Op]


def _scalar(v: str):
    if v in ("True", "False"):
        return v == "True"
    if (v[0] != "-" and not v[0].isdigit()) or (v[0] == "-" and len(v) > 1 and not v[1].isdigit()):
        return v
    if "." in v or "e" in v:
        return float(v)
    return int(v)


def parse_value(v: str):
    if v in ("None", "()", "[]"):
        return None
    if v[0] in "([":
        return [_scalar(e) for e in v[1:-1].split(",")]
    return _scalar(v)


def _shape(v: str):
    close = v.rfind(")")
    dims = tuple(int(e) if e not in ("?",) else -1 for e in v[1:close].split(",") if e != "")
    return dims, v[close + 1:]


def load(param_path: str) -> Graph:
    with open(param_path) as f:
        lines = [ln.rstrip("\n") for ln in f]
    n_ops = int(lines[1].split()[0])
    ops = []
    for ln in lines[2:2 + n_ops]:
        tok = ln.split()
        t, name, nin, nout = tok[0], tok[1], int(tok[2]), int(tok[3])
        ins = tok[4:4 + nin]
        outs = tok[4 + nin:4 + nin + nout]
        op = Op(t, name, ins, outs)
        for item in tok[4 + nin + nout:]:
            key, _, val = item.partition("=")
            if key.startswith("@"):
                op.attrs[key[1:]] = _shape(val)
            elif key.startswith("#"):
                op.shapes[key[1:]] = _shape(val)
            elif key.startswith("$"):
                continue
            else:
                op.params[key] = parse_value(val)
        ops.append(op)
    return Graph(ops)


def read_weights(bin_path: str) -> Dict[str, np.ndarray]:
    """All fp32 attributes of a stored-zip .pnnx.bin, keyed '<op>.<attr>'."""
    out = {}
    with zipfile.ZipFile(bin_path) as z:
        for info in z.infolist():
            out[info.filename] = np.frombuffer(z.read(info), dtype="<f4").copy()
    return out


def shaped_weights(graph: Graph, flat: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    """Reshape the flat weights with the attribute shapes of the graph."""
    res = {}
    for op in graph.ops:
        for a, (shape, _) in op.attrs.items():
            key = f"{op.name}.{a}"
            if key in flat:
                res[key] = flat[key].reshape(shape)
    return res
