"""lotusinfer_b200: sm_100a dense-contraction kernels behind a C ABI.

The compute path is liblotus_b200.so (built by ``python -m lotusinfer_b200.build``);
``abi`` binds it with ctypes, ``kernels`` calls it per operator on torch-owned
device memory, ``graph`` drives the native PNNX Graph runtime.
"""
__version__ = "0.1.0"
