"""elffuss-engine_b200: the GGUF quantized GEMV/GEMM hot path of the Elffuss
engine, rebuilt for NVIDIA B200 (sm_100a).

The product is ``libelffuss_cuda.so`` (C ABI in ``include/elffuss_cuda.h``);
this package is its Python host: ``ops.QuantOps`` mirrors the reference's
``createQuantOps`` operator API, ``formats`` holds the block geometry and the
seeded synthetic tensors, ``build`` compiles the library in-tree.

The directory name contains a hyphen, so it is imported under the name
``elffuss_engine_b200`` (see ``__graft_entry__.package()``).
"""
from ._lib import EfError, header_symbols, lib  # noqa: F401

__all__ = ["EfError", "lib", "header_symbols"]
