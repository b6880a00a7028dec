"""The allocation-free decode GEMV (ef_gemv_noalloc) against the regular one.

ef_gemv_noalloc exists for callers that cannot allocate device memory -- code
running during CUDA-graph stream capture, decode loops that cannot take the
device synchronization of cudaMalloc/cudaFree, hosts whose memory belongs to
another allocator -- and keeps its per-call activation fragments in a 1 MiB
file-scope device array instead of growable context scratch. It is called here
through the C ABI, twice in a row with different types and shapes (the second
call reuses the array the first one filled), and each result must agree with
ef_gemv on the same inputs within the GEMV acceptance bound
max|err| <= 1e-3 * ||row||_2 * ||x||_2. Oversized k must be refused.

This file is collected last so that a run stopping at the first failure has
already run every other test.
"""
import ctypes

import pytest
import torch

from elffuss_engine_b200 import formats
from elffuss_engine_b200._lib import EF_OK, lib

pytestmark = pytest.mark.gpu
REL = 1e-3
EF_ERR_RANGE = -7


def _noalloc(w, x, M, y):
    s = torch.cuda.current_stream().cuda_stream
    return lib().ef_gemv_noalloc(w.h, ctypes.c_void_p(x.data_ptr()), M, ctypes.c_void_p(y.data_ptr()),
                                 ctypes.c_void_p(s))


def test_noalloc_matches_gemv_on_two_calls(ops):
    cases = [("Q4_K", 640, 4096, 3), ("Q6_K", 384, 8192, 16)]
    for i, (t, rows, k, M) in enumerate(cases):
        raw = formats.synth(t, rows, k, seed=100 + i)
        w = ops.load_weight(t, raw, rows, k)
        be, _ = formats.block_info(t)
        wd = ops.dequant(t, w, rows * k // be).reshape(rows, k).double()
        x = torch.randn(M, k, device="cuda", generator=torch.Generator("cuda").manual_seed(i))
        ref = ops.matmul(t, w, x, rows, k, M)          # the existing entry point (ef_gemv)
        y = torch.full((M, rows), float("nan"), device="cuda")
        assert _noalloc(w, x, M, y) == EF_OK
        torch.cuda.synchronize()
        tol = REL * torch.linalg.norm(x.double(), dim=1)[:, None] * torch.linalg.norm(wd, dim=1)[None, :]
        assert bool(torch.all((y.double() - ref.double()).abs() <= tol)), f"call {i}: {t} {rows}x{k} M={M}"


def test_noalloc_refuses_k_beyond_its_array(ops):
    rows, k = 16, 256 * 160          # Q6_K, 16 tokens: 32 B per k -> 40960 k > 1 MiB of fragments
    raw = formats.synth("Q6_K", rows, k, seed=1)
    w = ops.load_weight("Q6_K", raw, rows, k)
    x = torch.randn(16, k, device="cuda")
    y = torch.empty(16, rows, device="cuda")
    assert _noalloc(w, x, 16, y) == EF_ERR_RANGE
    assert _noalloc(w, x, 1, torch.empty(1, rows, device="cuda")) == EF_OK   # 1 token fits
