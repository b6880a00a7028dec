"""Generate the golden fixtures in this directory (run in the build container).

The reference (utopia-ia/elffuss-engine) ships no tests, fixtures or golden
vectors, and its arithmetic is WGSL for WebGPU, which cannot run here. The pins
are therefore:

* the i-quant codebooks of the reference, read as TEXT from its
  ``js/quant-tables.js`` (``IQ2XXS_GRID``, ``IQ1S_GRID``: u32 pairs, byte j of
  entry e is byte (j & 3) of word 2e + (j >> 2), quant-tables.js:34-36), stored
  here as sha256 digests plus the gguf-py 0.19.0 tables they must equal;
* block decodes produced by gguf-py 0.19.0 (``gguf.quants.dequantize``), the
  llama.cpp-family decoder the reference says it validates against
  (README.md:150-156), for seeded blocks of every hot-path type drawn with the
  BASELINE.json distributions plus hand-made edge blocks;
* small matrix products computed in numpy f64 from those gguf-py decodes.

Usage:  python tests/golden/make_golden.py --reference PATH
Writes: tests/golden/golden.npz
"""
from __future__ import annotations

import argparse
import hashlib
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

TYPES = {"Q8_0": (8, 32, 34), "Q4_K": (12, 256, 144), "Q6_K": (14, 256, 210),
         "IQ2_XXS": (16, 256, 66), "IQ1_S": (19, 256, 50), "Q4_0": (2, 32, 18),
         "Q5_K": (13, 256, 176), "Q2_K": (10, 256, 84)}      # (appended: earlier draws unchanged)


def ref_grid(path: str, name: str) -> np.ndarray:
    """Parse `export const NAME = new Uint32Array([...])` from the JS source."""
    src = open(path, encoding="utf-8").read()
    m = re.search(r"export const %s = new Uint32Array\(\[(.*?)\]\);" % name, src, re.S)
    assert m, name
    words = [int(w, 16) for w in re.findall(r"0x[0-9a-fA-F]+", m.group(1))]
    return np.array(words, dtype="<u4").view(np.uint8).view(np.int8).reshape(-1, 8)


def gguf_grid(name: str) -> np.ndarray:
    import gguf.quants as gq
    cls = getattr(gq, name)
    cls.init_grid()
    return np.rint(np.asarray(cls.grid, np.float32).reshape(-1, 8)).astype(np.int16).astype(np.int8)


def f16_bytes(v):
    return np.asarray(v, np.float16).view(np.uint8).reshape(-1, 2)


def blocks(name: str, nb: int, rng) -> np.ndarray:
    _, be, bb = TYPES[name]
    raw = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    if name == "Q8_0":          # d U[1e-3, 4e-3], q U[-127, 127] (config 0)
        raw[:, 0:2] = f16_bytes(rng.uniform(1e-3, 4e-3, nb))
        raw[:, 2:] = rng.integers(-127, 128, size=(nb, 32)).astype(np.int8).view(np.uint8)
    elif name == "Q4_K":        # d, dmin U[1e-4, 5e-4]; sc/m and nibbles uniform (config 1)
        raw[:, 0:2] = f16_bytes(rng.uniform(1e-4, 5e-4, nb))
        raw[:, 2:4] = f16_bytes(rng.uniform(1e-4, 5e-4, nb))
    elif name == "Q5_K":        # as Q4_K
        raw[:, 0:2] = f16_bytes(rng.uniform(1e-4, 5e-4, nb))
        raw[:, 2:4] = f16_bytes(rng.uniform(1e-4, 5e-4, nb))
    elif name == "Q2_K":        # d, dmin (at the end of the block) U[1e-4, 5e-4]
        raw[:, 80:82] = f16_bytes(rng.uniform(1e-4, 5e-4, nb))
        raw[:, 82:84] = f16_bytes(rng.uniform(1e-4, 5e-4, nb))
    elif name == "Q6_K":        # sc int8 U[-64, 63], d U[1e-4, 5e-4] (config 1)
        raw[:, 192:208] = rng.integers(-64, 64, size=(nb, 16)).astype(np.int8).view(np.uint8)
        raw[:, 208:210] = f16_bytes(rng.uniform(1e-4, 5e-4, nb))
    else:                       # Q4_0 / i-quants: d U[1e-3, 4e-3]
        raw[:, 0:2] = f16_bytes(rng.uniform(1e-3, 4e-3, nb))
    return raw


def edge_blocks(name: str) -> np.ndarray:
    """Hand-made blocks: extreme scales, negative/subnormal d, all sign paths."""
    _, be, bb = TYPES[name]
    out = []
    ds = [np.float16(1.0), np.float16(-0.5), np.float16(6.1e-5), np.float16(3e-7),  # subnormal
          np.float16(0.0), np.float16(65504.0)]
    for i, d in enumerate(ds):
        b = np.zeros(bb, np.uint8)
        if name == "Q6_K":
            b[:192] = (np.arange(192) * 37 + i) & 0xFF
            b[192:208] = np.array([-64, 63, -1, 0, 1, 127, -128, 5] * 2, np.int8).view(np.uint8)
            b[208:210] = np.frombuffer(d.tobytes(), np.uint8)
        elif name == "Q2_K":
            b[:80] = (np.arange(80) * 41 + 3 * i) & 0xFF
            b[80:82] = np.frombuffer(d.tobytes(), np.uint8)
            b[82:84] = np.frombuffer(np.float16(-d if i % 2 else d).tobytes(), np.uint8)
        elif name in ("Q4_K", "Q5_K"):
            b[0:2] = np.frombuffer(d.tobytes(), np.uint8)
            b[2:4] = np.frombuffer(np.float16(-d if i % 2 else d).tobytes(), np.uint8)
            b[4:16] = [0xFF, 0xC0, 0x3F, 0x80, 0x7F, 0xC1, 0x00, 0xFF, 0xA5, 0x5A, 0xF0, 0x0F]
            b[16:] = (np.arange(bb - 16) * 29 + i) & 0xFF
        elif name == "Q8_0":
            b[0:2] = np.frombuffer(d.tobytes(), np.uint8)
            b[2:] = np.array([-128, 127, -127, 0, 1, -1] * 6, np.int8)[:32].view(np.uint8)
        else:
            b[0:2] = np.frombuffer(d.tobytes(), np.uint8)
            b[2:] = (np.arange(bb - 2) * 53 + 7 * i) & 0xFF
        out.append(b)
    return np.stack(out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="the reference checkout (for js/quant-tables.js)")
    args = ap.parse_args()
    import gguf.quants as gq
    from gguf.constants import GGMLQuantizationType as GT

    rng = np.random.default_rng(20261201)
    fx = {}
    tables = os.path.join(args.reference, "js", "quant-tables.js")
    for js_name, py_name in (("IQ2XXS_GRID", "IQ2_XXS"), ("IQ1S_GRID", "IQ1_S")):
        r = ref_grid(tables, js_name)
        g = gguf_grid(py_name)
        assert np.array_equal(r, g), f"{js_name}: reference table differs from gguf-py"
        fx[f"grid_{py_name}"] = g
        fx[f"grid_{py_name}_sha256"] = np.frombuffer(
            hashlib.sha256(r.tobytes()).digest(), np.uint8)

    for name, (tid, be, bb) in TYPES.items():
        raw = np.concatenate([blocks(name, 48, rng), edge_blocks(name)])
        deq = gq.dequantize(raw.reshape(-1), GT[name]).astype(np.float32).reshape(-1)
        fx[f"{name}_raw"] = raw
        fx[f"{name}_deq_bits"] = deq.view(np.uint32)
        # A small product: rows x k with tokens 1 and 3, f64 from the gguf-py decode.
        rows, k = 8, 2 * be if be == 256 else 8 * be
        w = blocks(name, rows * k // be, rng)
        wd = gq.dequantize(w.reshape(-1), GT[name]).astype(np.float64).reshape(rows, k)
        x = rng.standard_normal((3, k)).astype(np.float32)
        fx[f"{name}_mm_w"] = w
        fx[f"{name}_mm_shape"] = np.array([rows, k])
        fx[f"{name}_mm_x"] = x
        fx[f"{name}_mm_y"] = x.astype(np.float64) @ wd.T
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **fx)
    print("wrote", os.path.join(HERE, "golden.npz"))


if __name__ == "__main__":
    main()
