"""Decode GEMV parity on the GPU: every hot-path type, 1..16 tokens, ragged
shapes, fused SwiGLU and sections, against the f64 CPU oracle within the
acceptance bound max|err| <= 1e-3 * ||row||_2 * ||x||_2.
At full benchmark sizes the check is against the exact product of the
oracle's dequantised weights (summed in f64 on the GPU) with the same bound."""
import numpy as np
import pytest
import torch

from elffuss_engine_b200 import formats

pytestmark = pytest.mark.gpu
REL = 1e-3   # acceptance tolerance (north_star)


def _check(oracle_mod, t, raw, rows, k, x, y):
    yr = oracle_mod.matmul_f64(t, raw, rows, k, x=x, tokens=x.shape[0])
    tol = oracle_mod.tolerance(t, raw, rows, k, x, rel=REL)
    err = np.abs(y.astype(np.float64) - yr)
    assert np.all(err <= tol), f"max err/tol = {(err / tol).max():.3f}"
    return (err / tol).max()


SHAPES = [("Q8_0", 128, 2048), ("Q8_0", 40, 96), ("Q4_0", 128, 2048), ("Q4_0", 24, 160),
          ("Q4_K", 256, 1024), ("Q4_K", 36, 4096), ("Q5_K", 128, 1024), ("Q5_K", 21, 2304),
          ("Q2_K", 128, 1024), ("Q2_K", 19, 2304),
          ("Q6_K", 128, 1024), ("Q6_K", 20, 2304), ("IQ2_XXS", 64, 1024), ("IQ1_S", 64, 1024)]


@pytest.mark.parametrize("t,rows,k", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 3, 4, 8, 9, 16])
def test_gemv_vs_oracle(ops, oracle_mod, t, rows, k, M):
    raw = formats.synth(t, rows, k, seed=M * 131 + rows)
    w = ops.load_weight(t, raw, rows, k)
    x = np.random.default_rng(M).standard_normal((M, k)).astype(np.float32)
    y = ops.matmul(t, w, torch.from_numpy(x).cuda(), rows, k, M).cpu().numpy()
    assert y.shape == (M, rows)
    _check(oracle_mod, t, raw, rows, k, x, y)


@pytest.mark.parametrize("t", formats.HOT_TYPES)
def test_gemv_is_deterministic(ops, t):
    rows, k = 512, 4096
    raw = formats.synth(t, rows, k, seed=1)
    w = ops.load_weight(t, raw, rows, k)
    x = torch.randn(3, k, device="cuda")
    a = ops.matmul(t, w, x, rows, k, 3)
    b = ops.matmul(t, w, x, rows, k, 3)
    assert torch.equal(a, b)


@pytest.mark.parametrize("t", ["Q8_0", "Q4_K", "Q6_K"])
@pytest.mark.parametrize("M", [1, 16])
def test_swiglu_vs_oracle(ops, oracle_mod, t, M):
    rows, k = 160, 1024
    rg, ru = formats.synth(t, rows, k, seed=5), formats.synth(t, rows, k, seed=6)
    wg, wu = ops.load_weight(t, rg, rows, k), ops.load_weight(t, ru, rows, k)
    x = np.random.default_rng(2).standard_normal((M, k)).astype(np.float32)
    y = ops.gemv.gateUp(t, wg, wu, torch.from_numpy(x).cuda(), rows, k, M).cpu().numpy()
    g = oracle_mod.matmul_f64(t, rg, rows, k, x=x, tokens=M)
    u = oracle_mod.matmul_f64(t, ru, rows, k, x=x, tokens=M)
    want = oracle_mod.swiglu_f64(g, u)
    # error propagation of silu(g)*u from the two GEMV bounds
    tg = oracle_mod.tolerance(t, rg, rows, k, x, rel=REL)
    tu = oracle_mod.tolerance(t, ru, rows, k, x, rel=REL)
    dsilu = 1.1 * np.abs(u) + 1e-30
    tol = dsilu * tg + (np.abs(g) + 1.0) * tu
    assert np.all(np.abs(y - want) <= tol)


@pytest.mark.parametrize("t", ["Q8_0", "Q4_K"])
@pytest.mark.parametrize("M", [2, 4])
def test_sections_equal_single(ops, oracle_mod, t, M):
    """Several matrices in one launch give each matrix's product: within the
    bound against the oracle, and bit-equal to single calls."""
    k = 1024
    shapes = [512, 128, 128, 32]
    raws = [formats.synth(t, r, k, seed=i) for i, r in enumerate(shapes)]
    ws = [ops.load_weight(t, raw, r, k) for raw, r in zip(raws, shapes)]
    x = torch.randn(M, k, device="cuda", generator=torch.Generator("cuda").manual_seed(M))
    ys = ops.gemv.secciones(t, ws, x, shapes, k, M)
    xn = x.cpu().numpy()
    for w, raw, r, y in zip(ws, raws, shapes, ys):
        _check(oracle_mod, t, raw, r, k, xn, y.cpu().numpy())
        single = ops.gemv.matmul(t, w, x, r, k, M)
        torch.testing.assert_close(y, single, rtol=0, atol=0)
    assert ops.gemv.despachados()["secciones"] >= 1


@pytest.mark.parametrize("t,rows,k", [("Q8_0", 8192, 2048), ("Q4_K", 14336, 4096), ("Q4_K", 4096, 14336),
                                      ("Q6_K", 14336, 4096), ("Q6_K", 4096, 14336)])
@pytest.mark.parametrize("M", [1, 4, 16])
def test_full_size_vs_oracle(ops, parity_report, t, rows, k, M):
    """Benchmark shapes (configs 0 and 1): the GEMV against the exact product
    of the oracle's f32 dequantisation (the C restatement, not the library's
    own dequant) and the f32 x, summed in f64 on the GPU, within the bound."""
    from oracle.forward_f32 import load_matrix
    raw = formats.synth(t, rows, k, seed=42)
    w = ops.load_weight(t, raw, rows, k)
    x = torch.randn(M, k, device="cuda", generator=torch.Generator("cuda").manual_seed(M))
    y = ops.matmul(t, w, x, rows, k, M).double()
    wd = load_matrix(raw, rows, k, t, "cuda", torch.float64)
    ref = x.double() @ wd.T
    tol = REL * torch.linalg.norm(x.double(), dim=1)[:, None] * torch.linalg.norm(wd, dim=1)[None, :]
    ratio = float(((y - ref).abs() / tol).max())
    parity_report[f"gemv {t} {rows}x{k} M={M}"] = round(ratio, 5)
    assert ratio <= 1.0


def test_wrong_weight_raises(ops):
    from elffuss_engine_b200 import EfError
    raw = formats.synth("Q4_K", 16, 256, seed=0)
    w = ops.load_weight("Q4_K", raw, 16, 256)
    with pytest.raises(EfError):
        ops.matmul("Q6_K", w, torch.randn(1, 256, device="cuda"), 16, 256, 1)
    with pytest.raises(EfError):
        ops.matmul("Q4_K", w, torch.randn(1, 256, device="cuda"), 32, 256, 1)
    with pytest.raises(EfError):
        ops.matmul("Q4_0X", w, torch.randn(1, 256, device="cuda"), 16, 256, 1)

