"""Python face of the CPU restatement in ``elffuss_oracle.c``.

TEST INFRASTRUCTURE: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use this module,
always as the checker. The product (the CUDA library and its Python host) never
imports it.

The i-quant codebooks handed to the C code come from gguf-py 0.19.0
(``gguf.quants.IQ2_XXS`` / ``IQ1_S``), an implementation independent of this
repository's generated CUDA header; both are pinned to the reference's
``js/quant-tables.js`` by the table hashes stored in ``tests/golden``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

# ggml type ids (reference js/gguf.js:48-64)
F32, F16, Q4_0, Q8_0, Q2_K, Q4_K, Q5_K, Q6_K, IQ2_XXS, IQ1_S = 0, 1, 2, 8, 10, 12, 13, 14, 16, 19
TYPE_IDS = {"F32": F32, "F16": F16, "Q4_0": Q4_0, "Q8_0": Q8_0, "Q2_K": Q2_K, "Q4_K": Q4_K, "Q5_K": Q5_K,
            "Q6_K": Q6_K, "IQ2_XXS": IQ2_XXS, "IQ1_S": IQ1_S}
BLOCK = {Q4_0: (32, 18), Q8_0: (32, 34), Q2_K: (256, 84), Q4_K: (256, 144), Q5_K: (256, 176),
         Q6_K: (256, 210), IQ2_XXS: (256, 66), IQ1_S: (256, 50)}

_lib = None


def build() -> str:
    """Compile liboracle.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.or_dequant.argtypes = [I, P, I64, P, P]
        L.or_matmul_f64.argtypes = [I, P, I64, I64, P, P, P, I64, I, P, I]
        L.or_matmul_f32.argtypes = [I, P, I64, I64, P, P, I64, P, I]
        L.or_row_norms.argtypes = [I, P, I64, I64, P, P]
        L.or_f32_to_f16_array.argtypes = [P, P, I64]
        L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_f16_to_f32.restype = ctypes.c_float
        L.or_f32_to_f16.argtypes = [ctypes.c_float]
        L.or_f32_to_f16.restype = ctypes.c_uint16
        L.or_swiglu_f64.argtypes = [P, P, I64, P]
        _lib = L
    return _lib


def type_id(t) -> int:
    return TYPE_IDS[t] if isinstance(t, str) else int(t)


_grids: dict = {}


def grid(t) -> np.ndarray:
    """The codebook of an i-quant type as int8 [entries, 8] (gguf-py 0.19.0)."""
    t = type_id(t)
    if t not in (IQ2_XXS, IQ1_S):
        return np.zeros((1, 8), np.int8)
    if t not in _grids:
        import gguf.quants as gq
        cls = gq.IQ2_XXS if t == IQ2_XXS else gq.IQ1_S
        cls.init_grid()
        g = np.asarray(cls.grid, dtype=np.float32).reshape(-1, 8)
        _grids[t] = np.ascontiguousarray(np.rint(g).astype(np.int16).astype(np.int8))
    return _grids[t]


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def dequant(t, raw: np.ndarray) -> np.ndarray:
    """All blocks of ``raw`` (GGUF bytes) to f32 (kernels.wgsl.js dequantShader)."""
    t = type_id(t)
    be, bb = BLOCK[t]
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    nb = raw.size // bb
    out = np.empty(nb * be, np.float32)
    g = grid(t)
    rc = lib().or_dequant(t, _p(raw), nb, _p(g), _p(out))
    assert rc == 0
    return out


def matmul_f64(t, raw, rows: int, k: int, x=None, xh=None, tokens: int = 1,
               w16: bool = False, threads: int = 0) -> np.ndarray:
    """y[tokens][rows] in f64. ``x`` f32 [tokens][k] or ``xh`` f16 bits (uint16)."""
    t = type_id(t)
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    y = np.empty((tokens, rows), np.float64)
    g = grid(t)
    xp = _p(np.ascontiguousarray(x, np.float32)) if x is not None else None
    xa = np.ascontiguousarray(x, np.float32) if x is not None else None
    xha = np.ascontiguousarray(xh, np.uint16) if xh is not None else None
    rc = lib().or_matmul_f64(t, _p(raw), rows, k, _p(g),
                             _p(xa) if xa is not None else None,
                             _p(xha) if xha is not None else None,
                             tokens, 1 if w16 else 0, _p(y), threads or (os.cpu_count() or 1))
    del xp
    assert rc == 0
    return y


def matmul_f32(t, raw, rows: int, k: int, x, tokens: int = 1, threads: int = 1) -> np.ndarray:
    """y[tokens][rows] accumulated in f32 in natural k order (the timed CPU path)."""
    t = type_id(t)
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    xa = np.ascontiguousarray(x, np.float32)
    y = np.empty((tokens, rows), np.float32)
    rc = lib().or_matmul_f32(t, _p(raw), rows, k, _p(grid(t)), _p(xa), tokens, _p(y), threads)
    assert rc == 0
    return y


def row_norms(t, raw, rows: int, k: int) -> np.ndarray:
    t = type_id(t)
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    out = np.empty(rows, np.float64)
    assert lib().or_row_norms(t, _p(raw), rows, k, _p(grid(t)), _p(out)) == 0
    return out


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f16 bits (cpu.js:84-99), as uint16."""
    xa = np.ascontiguousarray(x, np.float32).reshape(-1)
    out = np.empty(xa.size, np.uint16)
    lib().or_f32_to_f16_array(_p(xa), _p(out), xa.size)
    return out.reshape(np.shape(x))


def swiglu_f64(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float64)
    u = np.ascontiguousarray(u, np.float64)
    out = np.empty_like(g)
    lib().or_swiglu_f64(_p(g), _p(u), g.size, _p(out))
    return out


def tolerance(t, raw, rows: int, k: int, x: np.ndarray, rel: float = 1e-3) -> np.ndarray:
    """Per-(token,row) bound rel * ||row||_2 * ||x_t||_2 of the acceptance test."""
    rn = row_norms(t, raw, rows, k)
    xn = np.linalg.norm(np.asarray(x, np.float64).reshape(-1, k), axis=1)
    return rel * xn[:, None] * rn[None, :]
