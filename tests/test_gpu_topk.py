"""The device top-k of the sampler (ef_topk, kernels.topk.wgsl.js): exactly
the m first logits by (larger value, lower index), -0 equal to +0, the
logits' own bits, several rows, rows shorter than m, and the NaN flag."""
import ctypes

import numpy as np
import pytest
import torch

from elffuss_engine_b200._lib import EfError, check, lib

pytestmark = pytest.mark.gpu


def P(t):
    return ctypes.c_void_p(t.data_ptr())


def _topk(ops, logits, m):
    rows, n = logits.shape
    ids = torch.empty(rows, m, dtype=torch.int32, device="cuda")
    vals = torch.empty(rows, m, device="cuda")
    flags = torch.empty(rows, dtype=torch.int32, device="cuda")
    h = ops.ctx.bind()
    check(lib().ef_topk(h, P(logits), rows, n, m, P(ids), P(vals), P(flags)), h)
    return ids.cpu().numpy(), vals.cpu().numpy(), flags.cpu().numpy()


def _want(row, m):
    order = np.lexsort((np.arange(row.size), -row.astype(np.float64)))   # value desc, then index asc
    return order[:m]


@pytest.mark.parametrize("n,m", [(70000, 40), (128256, 256), (4096, 1), (100, 64)])
def test_topk_exact_order_and_bits(ops, n, m):
    g = torch.Generator("cuda").manual_seed(n + m)
    lg = torch.randn(3, n, device="cuda", generator=g)
    lg[0, 10:20] = 3.5                      # ties: the lower indices first
    lg[0, n - 5:] = 3.5
    lg[1, 7] = -0.0                         # -0 and +0 are equal: index order
    lg[1, 3] = 0.0
    lg[1, :] = torch.where(lg[1] > 0, lg[1] * 0 - 1.0, lg[1])   # the zeros are now the largest
    lg[1, 7] = -0.0
    lg[1, 3] = 0.0
    ids, vals, flags = _topk(ops, lg, m)
    host = lg.cpu().numpy()
    for r in range(3):
        want = _want(host[r], m)
        k = min(m, n)
        assert ids[r, :k].tolist() == want.tolist()
        assert np.array_equal(vals[r, :k].view(np.uint32), host[r, want].view(np.uint32))
        assert flags[r] == 0
    if m >= 2:
        assert ids[1, 0] == 3 and ids[1, 1] == 7 and np.signbit(vals[1, 1])


def test_topk_short_rows_and_nan_flag(ops):
    lg = torch.randn(2, 50, device="cuda")
    lg[1, 17] = float("nan")
    ids, vals, flags = _topk(ops, lg, 64)
    assert flags.tolist() == [0, 2]
    assert ids[0, :50].tolist() == _want(lg[0].cpu().numpy(), 50).tolist()
    assert (ids[0, 50:] == -1).all()


def test_topk_limits(ops):
    lg = torch.randn(1, 1000, device="cuda")
    with pytest.raises(EfError):
        _topk(ops, lg, 300)
