"""Host-side logic that needs no GPU: formats, generators, planners, errors."""
import numpy as np
import pytest

from elffuss_engine_b200 import formats
from elffuss_engine_b200.ops import Gemm2Ops


@pytest.mark.parametrize("t", formats.HOT_TYPES)
def test_synth_sizes_and_seeds(t):
    rows, k = 16, 512
    a = formats.synth(t, rows, k, seed=1)
    b = formats.synth(t, rows, k, seed=1)
    c = formats.synth(t, rows, k, seed=2)
    assert a.size == formats.tensor_bytes(t, rows, k)
    assert np.array_equal(a, b) and not np.array_equal(a, c)


def test_synth_distributions(oracle_mod):
    raw = formats.synth("Q8_0", 64, 2048, seed=0).reshape(-1, 34)
    d = raw[:, :2].copy().view(np.float16).astype(np.float32)
    q = raw[:, 2:].view(np.int8)
    assert 1e-3 * (1 - 2 ** -10) <= d.min() and d.max() <= 4e-3 * (1 + 2 ** -10)
    assert q.min() >= -127 and q.max() <= 127
    raw6 = formats.synth("Q6_K", 16, 4096, seed=0).reshape(-1, 210)
    sc = raw6[:, 192:208].view(np.int8)
    assert sc.min() >= -64 and sc.max() <= 63


def test_quantize_q8_0_roundtrip(oracle_mod):
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((8, 256)) * 0.02).astype(np.float32)
    raw = formats.quantize_q8_0(w)
    back = oracle_mod.dequant("Q8_0", raw).reshape(8, 256)
    d = np.abs(w.reshape(-1, 32)).max(axis=1) / 127          # f32 scale used to round
    dh = d.astype(np.float16).astype(np.float32)             # stored f16 scale
    err = np.abs(back - w).reshape(-1, 32).max(axis=1)
    assert np.all(err <= 0.5 * d * 1.001 + 127 * np.abs(d - dh) + 1e-9)


def test_bad_k_raises():
    with pytest.raises(ValueError):
        formats.tensor_bytes("Q4_K", 4, 100)


def test_gemm2_plan_is_pure():
    assert Gemm2Ops.plan("Q8_0", 8192, 2048, 1) is None       # decode: GEMV
    assert Gemm2Ops.plan("Q8_0", 8192, 2048, 16) is None
    p = Gemm2Ops.plan("Q8_0", 8192, 2048, 512)
    assert p["via"] == "gemm" and p["bpr"] == 64
    assert Gemm2Ops.plan("Q4_K", 16, 100 * 256 + 1, 512) is None
