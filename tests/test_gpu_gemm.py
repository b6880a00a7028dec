"""Prefill GEMM parity: f16 activations, f32 accumulate, against the oracle's
GEMM2 contract (X rounded to f16; W rounded to f16 as the reference tile does,
kernels.gemm2.wgsl.js:12-23), within max|err| <= 1e-3 * ||row|| * ||x||."""
import numpy as np
import pytest
import torch

from elffuss_engine_b200 import formats

pytestmark = pytest.mark.gpu
REL = 1e-3


@pytest.mark.parametrize("t,rows,k", [("Q8_0", 256, 512), ("Q8_0", 48, 2048), ("Q8_0", 64, 640),
                                      ("Q8_0", 32, 4128), ("Q4_0", 256, 512), ("Q4_0", 40, 2048),
                                      ("Q4_0", 40, 4128), ("Q4_K", 128, 1024), ("Q4_K", 37, 2304),
                                      ("Q6_K", 64, 512), ("Q6_K", 37, 2304), ("Q5_K", 48, 1024),
                                      ("Q5_K", 37, 2304), ("Q2_K", 64, 512), ("Q2_K", 37, 2304),
                                      ("IQ2_XXS", 64, 512), ("IQ2_XXS", 37, 2304), ("IQ1_S", 64, 512),
                                      ("IQ1_S", 37, 2304)])
@pytest.mark.parametrize("M", [17, 64, 130])
def test_gemm_f16x_vs_oracle(ops, oracle_mod, t, rows, k, M):
    raw = formats.synth(t, rows, k, seed=M + rows)
    w = ops.load_weight(t, raw, rows, k)
    x = np.random.default_rng(M).standard_normal((M, k)).astype(np.float32)
    xh = oracle_mod.f32_to_f16_bits(x)
    y = ops.gemm2.matmul(t, w, torch.from_numpy(xh.view(np.float16)).cuda(), rows, k, M, x_f16=True)
    y = y.cpu().numpy()
    ops.gemm2.status()
    want = oracle_mod.matmul_f64(t, raw, rows, k, xh=xh, tokens=M, w16=True)
    tol = oracle_mod.tolerance(t, raw, rows, k, xh.view(np.float16).astype(np.float32), rel=REL)
    assert np.all(np.abs(y - want) <= tol)


def _exact(raw, t, rows, k):
    """The oracle's exact f32 dequantisation, as f64 on the GPU."""
    from oracle.forward_f32 import load_matrix
    return load_matrix(raw, rows, k, t, "cuda", torch.float64)


def _ratio(y, x, wd):
    """max |y - x wd^T| / (REL ||x_t|| ||row||), the reference product in f64."""
    ref = x.double() @ wd.T
    tol = REL * torch.linalg.norm(x.double(), dim=1)[:, None] * torch.linalg.norm(wd, dim=1)[None, :]
    return float(((y.double() - ref).abs() / tol).max())


@pytest.mark.parametrize("t,M,k,rows", [("Q8_0", 512, 2048, 8192), ("Q8_0", 2048, 8192, 2048),
                                        ("Q4_0", 512, 2048, 8192), ("Q4_K", 512, 4096, 4096),
                                        ("Q6_K", 512, 4096, 4096), ("Q5_K", 512, 4096, 4096),
                                        ("Q2_K", 512, 4096, 4096), ("IQ2_XXS", 512, 4096, 4096),
                                        ("IQ1_S", 512, 4096, 4096)])
def test_gemm_config2_vs_oracle(ops, parity_report, t, M, k, rows):
    """Config-2 shapes (f16 activations): the tcgen05 GEMM against the exact
    product of the oracle's dequantised weights and the same f16 x."""
    raw = formats.synth(t, rows, k, seed=2)
    w = ops.load_weight(t, raw, rows, k)
    x = torch.randn(M, k, device="cuda", generator=torch.Generator("cuda").manual_seed(3)).half()
    y = ops.gemm2.matmul(t, w, x, rows, k, M, x_f16=True)
    ops.gemm2.status()
    r = _ratio(y, x, _exact(raw, t, rows, k))
    parity_report[f"gemm f16x {t} M={M} K={k} N={rows}"] = round(r, 5)
    assert r <= 1.0


@pytest.mark.parametrize("t,rows,k", [("Q8_0", 2048, 2048), ("Q4_K", 1024, 4096), ("Q6_K", 1024, 4096),
                                      ("Q4_0", 512, 2048), ("Q5_K", 512, 2048), ("Q2_K", 512, 2048),
                                      ("IQ2_XXS", 512, 2048), ("IQ1_S", 512, 2048)])
@pytest.mark.parametrize("M", [17, 33, 63, 130])
def test_matmul_f32_x_prefill_vs_oracle(ops, parity_report, t, rows, k, M):
    """quant.matmul with f32 activations above 16 tokens (js/ops.js:827-1101):
    the f32 -> f16 conversion kernel, then the tcgen05 GEMM, against the exact
    f32 product of the oracle's weights and the unrounded x. The reference
    runs 17-63 tokens through its f32 tiled GEMM (kernels.gemm.wgsl.js:172)
    and 64+ through GEMM2 with f16 x; this path rounds x and the weights to
    f16 at every size, which the bound covers."""
    raw = formats.synth(t, rows, k, seed=M)
    w = ops.load_weight(t, raw, rows, k)
    x = torch.randn(M, k, device="cuda", generator=torch.Generator("cuda").manual_seed(M))
    y = ops.matmul(t, w, x, rows, k, M)
    ops.gemm2.status()
    r = _ratio(y, x, _exact(raw, t, rows, k))
    parity_report[f"matmul f32x {t} {rows}x{k} M={M}"] = round(r, 5)
    assert r <= 1.0


def test_cola_matches_batch_row(ops):
    rows, k, lote = 256, 1024, 64
    raw = formats.synth("Q8_0", rows, k, seed=4)
    w = ops.load_weight("Q8_0", raw, rows, k)
    x = torch.randn(lote, k, device="cuda")
    yb = ops.gemm2.matmul("Q8_0", w, x, rows, k, lote)
    y1 = ops.gemm2.cola("Q8_0", w, x[-1:].clone(), rows, k, lote)
    assert ops.gemm2.reproducible("Q8_0", rows, k, lote)
    torch.testing.assert_close(y1[0], yb[-1], rtol=0, atol=0)


@pytest.mark.parametrize("t,M,k,rows", [("Q8_0", 512, 2048, 8192), ("Q4_K", 512, 4096, 4096),
                                        ("Q6_K", 512, 4096, 4096)])
def test_gemm_repeatable(ops, t, M, k, rows):
    """The pipeline hands every weight stage back only after it is consumed:
    back-to-back calls on the same inputs give bit-identical outputs."""
    raw = formats.synth(t, rows, k, seed=3)
    w = ops.load_weight(t, raw, rows, k)
    x = torch.randn(M, k, device="cuda").half()
    y0 = ops.gemm2.matmul(t, w, x, rows, k, M, x_f16=True)
    for _ in range(10):
        assert torch.equal(ops.gemm2.matmul(t, w, x, rows, k, M, x_f16=True), y0)
    ops.gemm2.status()


def test_gemm_wait_timeout_is_reported_and_recovers(ops, oracle_mod):
    """Every pipeline wait given a limit of zero polls gives up at once: the
    kernel still drains its own copies and MMAs, frees its tensor memory and
    exits; ef_gemm_status reports EF_ERR_TIMEOUT; with the default limit back,
    the next GEMM matches the oracle's GEMM2 contract."""
    from elffuss_engine_b200._lib import EfError, check, lib
    t, rows, k, M = "Q8_0", 256, 2048, 130
    raw = formats.synth(t, rows, k, seed=11)
    w = ops.load_weight(t, raw, rows, k)
    x = np.random.default_rng(11).standard_normal((M, k)).astype(np.float32)
    xh = oracle_mod.f32_to_f16_bits(x)
    xd = torch.from_numpy(xh.view(np.float16)).cuda()
    h = ops.ctx.bind()
    try:
        check(lib().ef_gemm_set_wait_limit(h, 0), h)   # zero polls: every pipeline wait gives up at once
        ops.gemm2.matmul(t, w, xd, rows, k, M, x_f16=True)
        with pytest.raises(EfError) as err:
            ops.gemm2.status()
        assert "EF_ERR_TIMEOUT" in str(err.value)
    finally:
        check(lib().ef_gemm_set_wait_limit(h, -1), h)   # the default limit again
    ops.gemm2.status()   # cleared by the report above
    y = ops.gemm2.matmul(t, w, xd, rows, k, M, x_f16=True).cpu().numpy()
    ops.gemm2.status()
    want = oracle_mod.matmul_f64(t, raw, rows, k, xh=xh, tokens=M, w16=True)
    tol = oracle_mod.tolerance(t, raw, rows, k, xh.view(np.float16).astype(np.float32), rel=REL)
    assert np.all(np.abs(y - want) <= tol)
