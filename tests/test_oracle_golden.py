"""The CPU oracle against the golden fixtures (gguf-py decodes, reference tables).

The oracle is the checker of every GPU parity test, so it is pinned first:
its block decoders must reproduce gguf-py 0.19.0 bit for bit, its codebooks
must be the reference's js/quant-tables.js tables, and its f64 product must
reproduce the fixture products.
"""
import hashlib

import numpy as np
import pytest

TYPES = ["Q8_0", "Q4_K", "Q6_K", "IQ2_XXS", "IQ1_S", "Q4_0", "Q5_K", "Q2_K"]


@pytest.mark.parametrize("t", TYPES)
def test_dequant_bit_exact_vs_golden(oracle_mod, golden, t):
    raw = golden[f"{t}_raw"]
    got = oracle_mod.dequant(t, raw)
    want = golden[f"{t}_deq_bits"]
    assert got.size == want.size
    np.testing.assert_array_equal(got.view(np.uint32), want)


@pytest.mark.parametrize("t", ["IQ2_XXS", "IQ1_S"])
def test_grids_are_reference_tables(oracle_mod, golden, t):
    g = oracle_mod.grid(t)
    np.testing.assert_array_equal(g, golden[f"grid_{t}"])
    digest = np.frombuffer(hashlib.sha256(np.ascontiguousarray(g).tobytes()).digest(), np.uint8)
    np.testing.assert_array_equal(digest, golden[f"grid_{t}_sha256"])


@pytest.mark.parametrize("t", TYPES)
def test_matmul_f64_vs_golden(oracle_mod, golden, t):
    rows, k = (int(v) for v in golden[f"{t}_mm_shape"])
    x = golden[f"{t}_mm_x"]
    y = oracle_mod.matmul_f64(t, golden[f"{t}_mm_w"], rows, k, x=x, tokens=x.shape[0])
    np.testing.assert_allclose(y, golden[f"{t}_mm_y"], rtol=1e-12, atol=1e-12)


def test_f16_rounding_matches_numpy(oracle_mod):
    rng = np.random.default_rng(3)
    v = np.concatenate([rng.standard_normal(10000).astype(np.float32) * 10,
                        np.array([65504, 65520, 1e-8, 6e-8, -0.0, np.inf, 2.0 ** -25], np.float32)])
    np.testing.assert_array_equal(oracle_mod.f32_to_f16_bits(v), v.astype(np.float16).view(np.uint16))


def test_f32_matmul_close_to_f64(oracle_mod, golden):
    t = "Q4_K"
    rows, k = (int(v) for v in golden[f"{t}_mm_shape"])
    x = golden[f"{t}_mm_x"]
    y32 = oracle_mod.matmul_f32(t, golden[f"{t}_mm_w"], rows, k, x, tokens=3, threads=2)
    tol = oracle_mod.tolerance(t, golden[f"{t}_mm_w"], rows, k, x)
    assert np.all(np.abs(y32 - golden[f"{t}_mm_y"]) <= tol)
