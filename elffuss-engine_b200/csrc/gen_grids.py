"""Write gen/iq_grids.h: the IQ2_XXS / IQ1_S codebooks for the CUDA library.

The codebooks are data of the GGUF format (ggml's iq2xxs_grid / iq1s_grid,
MIT-licensed; the reference carries them in js/quant-tables.js:40,107). They are
taken at build time from the installed gguf-py 0.19.0 package and emitted both
as raw bytes and as f16 bit patterns (the form the GEMV kernels stage into
shared memory). The header is a build product (git-ignored).
"""
from __future__ import annotations

import os
import sys

import numpy as np

MIT = """/*
 * Grid tables iq2xxs_grid and iq1s_grid of the GGUF format, generated from
 * gguf-py 0.19.0 (ggml). Those tables are distributed under the MIT License:
 *
 *   MIT License
 *
 *   Copyright (c) 2023-2026 The ggml authors
 *
 *   Permission is hereby granted, free of charge, to any person obtaining a copy
 *   of this software and associated documentation files (the "Software"), to deal
 *   in the Software without restriction, including without limitation the rights
 *   to use, copy, modify, merge, publish, distribute, sublicense, and/or sell
 *   copies of the Software, and to permit persons to whom the Software is
 *   furnished to do so, subject to the following conditions:
 *
 *   The above copyright notice and this permission notice shall be included in all
 *   copies or substantial portions of the Software.
 *
 *   THE SOFTWARE IS PROVIDED "AS IS", WITHOUT WARRANTY OF ANY KIND, EXPRESS OR
 *   IMPLIED, INCLUDING BUT NOT LIMITED TO THE WARRANTIES OF MERCHANTABILITY,
 *   FITNESS FOR A PARTICULAR PURPOSE AND NONINFRINGEMENT. IN NO EVENT SHALL THE
 *   AUTHORS OR COPYRIGHT HOLDERS BE LIABLE FOR ANY CLAIM, DAMAGES OR OTHER
 *   LIABILITY, WHETHER IN AN ACTION OF CONTRACT, TORT OR OTHERWISE, ARISING FROM,
 *   OUT OF OR IN CONNECTION WITH THE SOFTWARE OR THE USE OR OTHER DEALINGS IN THE
 *   SOFTWARE.
 *
 * GENERATED FILE (gen_grids.py) -- do not edit.
 */
"""


def grids():
    import gguf.quants as gq
    out = {}
    for name in ("IQ2_XXS", "IQ1_S"):
        cls = getattr(gq, name)
        cls.init_grid()
        g = np.rint(np.asarray(cls.grid, np.float32).reshape(-1, 8)).astype(np.int16)
        out[name] = g
    return out


def emit(path: str) -> None:
    g = grids()
    lines = [MIT, "#pragma once", "#include <stdint.h>", ""]
    for name, sym in (("IQ2_XXS", "EF_GRID_IQ2XXS"), ("IQ1_S", "EF_GRID_IQ1S")):
        a = g[name]
        n = a.shape[0]
        lines.append(f"#define {sym}_ENTRIES {n}")
        # Initializer lists (macros) so that both host arrays and __device__
        # arrays can be defined from the same data.
        raw = a.astype(np.int8).reshape(-1)
        lines.append(f"#define {sym}_I8_INIT \\")
        for i in range(0, raw.size, 32):
            lines.append("  " + ",".join(str(int(v)) for v in raw[i:i + 32]) + ", \\")
        lines.append("")
        f16 = a.astype(np.float16).view(np.uint16).reshape(-1)
        lines.append(f"#define {sym}_F16_INIT \\")
        for i in range(0, f16.size, 16):
            lines.append("  " + ",".join("0x%04x" % int(v) for v in f16[i:i + 16]) + ", \\")
        lines.append("")
    lines.append("/* end of generated tables */")
    lines.append("")
    os.makedirs(os.path.dirname(path), exist_ok=True)
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        f.write("\n".join(lines))
    os.replace(tmp, path)


if __name__ == "__main__":
    emit(sys.argv[1] if len(sys.argv) > 1 else
         os.path.join(os.path.dirname(os.path.abspath(__file__)), "gen", "iq_grids.h"))
