"""Python handle on the native graph runtime (include/lotus_graph.h).

    g = Graph(param_path, bin_path, batch=256)
    g.set_input(host_nchw_f32)        # pinned host -> device, async on the graph stream
    g.forward()                       # enqueue (CUDA-graph replay after the first call)
    out = g.get_output()              # device -> host, waits

Mirrors lotus::Graph of the reference (include/graph.hpp:15-43).  All work is
done by liblotus_b200.so; this class only forwards pointers and streams.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import numpy as np

from . import abi
from .abi import LotusError

_V, _I, _S, _D = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_double
_I64P = ctypes.POINTER(ctypes.c_int64)
_IP = ctypes.POINTER(ctypes.c_int)
_FP = ctypes.POINTER(ctypes.c_float)

GRAPH_SIGNATURES = {
    "lotus_graph_create": (_V, [ctypes.c_char_p, ctypes.c_char_p, _I, _I, _I]),
    "lotus_graph_destroy": (None, [_V]),
    "lotus_graph_input_shape": (_I, [_V, _I64P, _IP]),
    "lotus_graph_output_shape": (_I, [_V, _I64P, _IP]),
    "lotus_graph_input_ptr": (_V, [_V]),
    "lotus_graph_output_ptr": (_V, [_V]),
    "lotus_graph_stream": (_V, [_V]),
    "lotus_graph_set_input": (_I, [_V, _V, _S, _V]),
    "lotus_graph_get_output": (_I, [_V, _V, _S, _V]),
    "lotus_graph_forward": (_I, [_V, _V]),
    "lotus_graph_forward_sync": (_I, [_V]),
    "lotus_graph_synchronize": (_I, [_V]),
    "lotus_graph_layer_count": (_I, [_V]),
    "lotus_graph_layer_name": (ctypes.c_char_p, [_V, _I]),
    "lotus_graph_layer_type": (ctypes.c_char_p, [_V, _I]),
    "lotus_graph_layer_flops": (_D, [_V, _I]),
    "lotus_graph_layer_bytes": (_D, [_V, _I]),
    "lotus_graph_launches_per_forward": (_I, [_V]),
    "lotus_graph_profile_layers": (_I, [_V, _I, _FP]),
    "lotus_graph_operand": (_V, [_V, ctypes.c_char_p, _IP, _I64P, _IP]),
    "lotus_graph_layer_weight": (_V, [_V, _I, ctypes.POINTER(ctypes.c_size_t)]),
    "lotus_graph_submit": (_I, [_V, _V, _V, _IP]),
    "lotus_graph_copy_stream": (_V, [_V, _I]),
    "lotus_graph_slot_output": (_V, [_V, _I]),
    "lotus_graph_activation_bytes": (_S, [_V]),
}

NO_CUDA_GRAPH = 1
NO_RESIDUAL_FUSION = 2
NO_S2D_STEM = 4
NO_POOL_FUSION = 8
NO_CONCAT_FUSION = 16
NO_MEMORY_PLAN = 32

_bound = False


def _lib():
    global _bound
    L = abi.lib()
    if not _bound:
        for name, (res, args) in GRAPH_SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _bound = True
    return L


def _cuda_copy(dst: int, src: int, nbytes: int) -> None:
    """Device copy through the CUDA runtime torch has already loaded (test/debug helper)."""
    import torch  # noqa: F401  (ensures libcudart is loaded)
    rt = ctypes.CDLL("libcudart.so.12")
    rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    err = rt.cudaMemcpy(ctypes.c_void_p(dst), ctypes.c_void_p(src), nbytes, 4)  # cudaMemcpyDefault
    if err != 0:
        raise RuntimeError(f"cudaMemcpy failed with {err}")


class Graph:
    def __init__(self, param_path: str, bin_path: str, batch: int, device: int = -1, cuda_graph: bool = True,
                 fuse_residual: bool = True, s2d_stem: bool = True, fuse_pool: bool = True, fuse_concat: bool = True,
                 plan_memory: bool = True):
        flags = ((0 if cuda_graph else NO_CUDA_GRAPH) | (0 if fuse_residual else NO_RESIDUAL_FUSION) |
                 (0 if s2d_stem else NO_S2D_STEM) | (0 if fuse_pool else NO_POOL_FUSION) |
                 (0 if fuse_concat else NO_CONCAT_FUSION) | (0 if plan_memory else NO_MEMORY_PLAN))
        L = _lib()
        h = L.lotus_graph_create(param_path.encode(), bin_path.encode(), int(batch), int(device), flags)
        if not h:
            raise LotusError(-1, abi.last_error())
        self._h = ctypes.c_void_p(h)
        self.batch = batch
        self.input_shape = self._shape(L.lotus_graph_input_shape)
        self.output_shape = self._shape(L.lotus_graph_output_shape)

    def _shape(self, fn) -> tuple:
        dims = (ctypes.c_int64 * 8)()
        nd = ctypes.c_int()
        abi.check(fn(self._h, dims, ctypes.byref(nd)))
        return tuple(int(dims[i]) for i in range(nd.value))

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib().lotus_graph_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------------- data
    @property
    def stream(self) -> int:
        return int(_lib().lotus_graph_stream(self._h) or 0)

    @property
    def input_ptr(self) -> int:
        return int(_lib().lotus_graph_input_ptr(self._h))

    @property
    def output_ptr(self) -> int:
        return int(_lib().lotus_graph_output_ptr(self._h))

    def set_input(self, host: np.ndarray, stream: Optional[int] = None) -> None:
        assert host.dtype == np.float32 and host.flags["C_CONTIGUOUS"] and host.shape == self.input_shape
        abi.check(_lib().lotus_graph_set_input(self._h, ctypes.c_void_p(host.ctypes.data), host.size,
                                               ctypes.c_void_p(stream) if stream else None))

    def set_input_ptr(self, host_ptr: int, count: int, stream: Optional[int] = None) -> None:
        abi.check(_lib().lotus_graph_set_input(self._h, ctypes.c_void_p(host_ptr), count,
                                               ctypes.c_void_p(stream) if stream else None))

    def get_output_into(self, host_ptr: int, count: int, stream: Optional[int] = None) -> None:
        abi.check(_lib().lotus_graph_get_output(self._h, ctypes.c_void_p(host_ptr), count,
                                                ctypes.c_void_p(stream) if stream else None))

    def submit(self, host_in_ptr: int, host_out_ptr: int) -> int:
        """Pipelined batch from host memory (lotus_graph_submit): returns the
        slot used; the host buffers must stay alive until synchronize()."""
        slot = ctypes.c_int()
        abi.check(_lib().lotus_graph_submit(self._h, ctypes.c_void_p(host_in_ptr), ctypes.c_void_p(host_out_ptr),
                                            ctypes.byref(slot)))
        return slot.value

    def copy_stream(self, which: int) -> int:
        s = _lib().lotus_graph_copy_stream(self._h, int(which))
        if not s:
            raise LotusError(-3, abi.last_error())
        return int(s)

    def slot_output(self, slot: int) -> int:
        return int(_lib().lotus_graph_slot_output(self._h, int(slot)))

    def forward(self, stream: Optional[int] = None) -> None:
        abi.check(_lib().lotus_graph_forward(self._h, ctypes.c_void_p(stream) if stream else None))

    def forward_sync(self) -> None:
        abi.check(_lib().lotus_graph_forward_sync(self._h))

    def get_output(self) -> np.ndarray:
        """Synchronous copy of the NCHW fp32 output (waits for the graph stream)."""
        out = np.empty(self.output_shape, np.float32)
        abi.check(_lib().lotus_graph_get_output(self._h, ctypes.c_void_p(out.ctypes.data), out.size, None))
        self.synchronize()
        return out

    def synchronize(self) -> None:
        abi.check(_lib().lotus_graph_synchronize(self._h))

    def run(self, x: np.ndarray) -> np.ndarray:
        """Reference-style one-shot inference: input, Forward(), Output()."""
        self.set_input(np.ascontiguousarray(x, np.float32))
        self.forward()
        return self.get_output()

    # ---------------------------------------------------------------- introspection
    def layers(self) -> List[dict]:
        L = _lib()
        out = []
        for i in range(L.lotus_graph_layer_count(self._h)):
            out.append({"name": L.lotus_graph_layer_name(self._h, i).decode(),
                        "type": L.lotus_graph_layer_type(self._h, i).decode(),
                        "flops": float(L.lotus_graph_layer_flops(self._h, i)),
                        "bytes": float(L.lotus_graph_layer_bytes(self._h, i))})
        return out

    def operand(self, name: str):
        """(device pointer, format, logical NCHW shape) of an operand, or None."""
        fmt = ctypes.c_int()
        dims = (ctypes.c_int64 * 8)()
        nd = ctypes.c_int()
        ptr = _lib().lotus_graph_operand(self._h, name.encode(), ctypes.byref(fmt), dims, ctypes.byref(nd))
        if not ptr:
            return None
        return int(ptr), int(fmt.value), tuple(int(dims[i]) for i in range(nd.value))

    def operand_array(self, name: str) -> "np.ndarray":
        """Copy of an operand as NCHW fp32 numpy (synchronises the graph stream)."""
        import torch
        ptr, fmt, shape = self.operand(name)
        self.synchronize()
        from . import kernels
        if fmt == 0:
            n = int(np.prod(shape))
            t = torch.empty(n, dtype=torch.float32, device="cuda")
            _cuda_copy(t.data_ptr(), ptr, n * 4)
            return t.view(shape).cpu().numpy()
        c = shape[1]
        sp = shape[2:] if len(shape) == 4 else (1, 1)
        cs = abi.channel_stride(c)
        n = shape[0] * sp[0] * sp[1] * cs
        t = torch.empty(n, dtype=torch.float16, device="cuda")
        _cuda_copy(t.data_ptr(), ptr, n * 2)
        return kernels.from_nhwc(t.view(shape[0], sp[0], sp[1], cs), c).reshape(shape).cpu().numpy()

    def layer_weight(self, i: int):
        """Copy of layer i's prepacked fp16 weight as a 1-D numpy array (or None)."""
        import torch
        nb = ctypes.c_size_t()
        ptr = _lib().lotus_graph_layer_weight(self._h, int(i), ctypes.byref(nb))
        if not ptr:
            return None
        self.synchronize()
        t = torch.empty(nb.value // 2, dtype=torch.float16, device="cuda")
        _cuda_copy(t.data_ptr(), int(ptr), nb.value)
        return t.cpu().numpy()

    def activation_bytes(self) -> int:
        return int(_lib().lotus_graph_activation_bytes(self._h))

    def launches_per_forward(self) -> int:
        return int(_lib().lotus_graph_launches_per_forward(self._h))

    def profile_layers(self, reps: int = 5) -> List[float]:
        n = _lib().lotus_graph_layer_count(self._h)
        ms = (ctypes.c_float * n)()
        abi.check(_lib().lotus_graph_profile_layers(self._h, int(reps), ms))
        return [float(v) for v in ms]
