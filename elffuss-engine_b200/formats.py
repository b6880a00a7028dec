"""GGUF block formats of the hot path and seeded synthetic tensors.

Block geometry follows the reference's type table (js/gguf.js:48-64,
js/kernels.wgsl.js:886-892). The generators draw raw block fields with the
distributions of the benchmark configurations (numpy, seeded):

* Q8_0: d = f16(U[1e-3, 4e-3]), qs int8 U[-127, 127]                 (config 0)
* Q4_K: d, dmin = f16(U[1e-4, 5e-4]); 6-bit scales/mins and nibbles uniform
        (all 12 scale bytes and 128 quant bytes uniform)               (config 1)
* Q6_K: ql, qh uniform bytes (6-bit quants uniform); int8 sc U[-64, 63];
        d = f16(U[1e-4, 5e-4])                                         (config 1)
* IQ2_XXS / IQ1_S: d = f16(U[1e-3, 4e-3]); grid indices, signs and block
        scales uniform random bits
* quantize_q8_0: f32 -> Q8_0 with d = max|x|/127, q = round-to-nearest-even(x/d)
  (configs 3-4: "quantized to Q8_0 (d = max|x|/127, round-to-nearest)").
"""
from __future__ import annotations

import numpy as np

from ._lib import TYPE_IDS, TYPE_NAMES

BLOCKS = {"Q4_0": (32, 18), "Q8_0": (32, 34), "Q2_K": (256, 84), "Q4_K": (256, 144), "Q5_K": (256, 176),
          "Q6_K": (256, 210), "IQ2_XXS": (256, 66), "IQ1_S": (256, 50)}
HOT_TYPES = ("Q8_0", "Q4_0", "Q2_K", "Q4_K", "Q5_K", "Q6_K", "IQ2_XXS", "IQ1_S")


def type_name(t) -> str:
    return TYPE_NAMES[t] if isinstance(t, int) else str(t)


def type_id(t) -> int:
    return TYPE_IDS[t] if isinstance(t, str) else int(t)


def block_info(t) -> tuple[int, int]:
    """(elements, bytes) of one block."""
    return BLOCKS[type_name(t)]


def tensor_bytes(t, rows: int, k: int) -> int:
    be, bb = block_info(t)
    if k % be:
        raise ValueError(f"{type_name(t)}: k={k} is not a multiple of {be}")
    return rows * (k // be) * bb


def _f16(rng, lo, hi, n):
    return rng.uniform(lo, hi, n).astype(np.float16).view(np.uint8).reshape(n, 2)


def synth(t, rows: int, k: int, seed: int = 0) -> np.ndarray:
    """Seeded raw GGUF bytes (uint8, rows * k/elems * bytes) of type `t`."""
    name = type_name(t)
    be, bb = block_info(name)
    if k % be:
        raise ValueError(f"{name}: k={k} is not a multiple of {be}")
    n = rows * (k // be)
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(n, bb), dtype=np.uint8)
    if name == "Q8_0":
        raw[:, 0:2] = _f16(rng, 1e-3, 4e-3, n)
        raw[:, 2:] = rng.integers(-127, 128, size=(n, 32), dtype=np.int8).view(np.uint8)
    elif name == "Q4_0":
        raw[:, 0:2] = _f16(rng, 1e-3, 4e-3, n)
    elif name in ("Q4_K", "Q5_K"):
        raw[:, 0:2] = _f16(rng, 1e-4, 5e-4, n)
        raw[:, 2:4] = _f16(rng, 1e-4, 5e-4, n)
    elif name == "Q2_K":                  # d, dmin at the end of the block
        raw[:, 80:82] = _f16(rng, 1e-4, 5e-4, n)
        raw[:, 82:84] = _f16(rng, 1e-4, 5e-4, n)
    elif name == "Q6_K":
        raw[:, 192:208] = rng.integers(-64, 64, size=(n, 16), dtype=np.int8).view(np.uint8)
        raw[:, 208:210] = _f16(rng, 1e-4, 5e-4, n)
    elif name in ("IQ2_XXS", "IQ1_S"):
        raw[:, 0:2] = _f16(rng, 1e-3, 4e-3, n)
    return raw.reshape(-1)


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """f32 [rows][k] -> Q8_0 bytes: d = max|x|/127 (f16), q = rne(x / d)."""
    w = np.asarray(w, np.float32)
    rows, k = w.shape
    if k % 32:
        raise ValueError("Q8_0 needs k % 32 == 0")
    blk = w.reshape(-1, 32)
    amax = np.abs(blk).max(axis=1)
    d = (amax / 127.0).astype(np.float32)
    dh = d.astype(np.float16)
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1.0), 0.0).astype(np.float32)
    q = np.clip(np.rint(blk * inv[:, None]), -127, 127).astype(np.int8)
    out = np.empty((blk.shape[0], 34), np.uint8)
    out[:, 0:2] = dh.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)
