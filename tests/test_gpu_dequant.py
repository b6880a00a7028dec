"""Bit-exact dequant and byte-exact repack round trip on the GPU, against the
CPU oracle (itself pinned to gguf-py and the reference tables)."""
import numpy as np
import pytest
import torch

from elffuss_engine_b200 import formats

pytestmark = pytest.mark.gpu

SHAPES = {  # rows x k, including ragged rows (not a multiple of 16) and partial chunks
    "Q8_0": [(16, 128), (37, 96), (8192 // 64, 2048), (5, 32 * 7)],
    "Q4_0": [(16, 128), (29, 96), (64, 2048), (3, 32 * 5)],
    "Q4_K": [(16, 256), (33, 768), (64, 4096)],
    "Q5_K": [(16, 256), (27, 768), (32, 4096)],
    "Q2_K": [(16, 256), (31, 512), (32, 4096)],
    "Q6_K": [(16, 256), (19, 512), (48, 4096)],
    "IQ2_XXS": [(16, 256), (21, 512)],
    "IQ1_S": [(16, 256), (23, 768)],
}
CASES = [(t, r, k) for t, shapes in SHAPES.items() for (r, k) in shapes]


@pytest.mark.parametrize("t,rows,k", CASES)
def test_dequant_bit_exact(ops, oracle_mod, t, rows, k):
    raw = formats.synth(t, rows, k, seed=rows * 7 + k)
    w = ops.load_weight(t, raw, rows, k)
    be, _ = formats.block_info(t)
    got = ops.dequant(t, w, rows * k // be).cpu().numpy()
    want = oracle_mod.dequant(t, raw)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("t,rows,k", CASES)
def test_repack_round_trip(ops, t, rows, k):
    raw = formats.synth(t, rows, k, seed=rows + k)
    w = ops.load_weight(t, raw, rows, k)
    back = w.unpack().cpu().numpy()
    np.testing.assert_array_equal(back, raw)


@pytest.mark.parametrize("t", ["Q8_0", "Q4_0", "Q4_K", "Q5_K", "Q2_K", "Q6_K", "IQ2_XXS", "IQ1_S"])
def test_golden_blocks_on_gpu(ops, golden, t):
    """The fixture's seeded + edge blocks (negative, subnormal, max scales) as a
    one-row-per-block tensor, decoded on the GPU vs gguf-py's bits."""
    raw = golden[f"{t}_raw"]
    be, bb = formats.block_info(t)
    nb = raw.shape[0]
    w = ops.load_weight(t, raw.reshape(-1), nb, be)
    got = ops.dequant(t, w, nb).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), golden[f"{t}_deq_bits"])


def test_load_from_device_bytes(ops, oracle_mod):
    rows, k = 40, 512
    raw = formats.synth("Q4_K", rows, k, seed=3)
    w = ops.load_weight("Q4_K", torch.from_numpy(raw).cuda(), rows, k)
    got = ops.dequant("Q4_K", w, rows * 2).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), oracle_mod.dequant("Q4_K", raw).view(np.uint32))


def test_slice_load_is_the_sub_matrix(ops, oracle_mod):
    rows, k = 64, 1024
    raw = formats.synth("Q6_K", rows, k, seed=9)
    full = oracle_mod.dequant("Q6_K", raw).reshape(rows, k)
    w = ops.load_weight_slice("Q6_K", raw, rows, k, 16, 24, 256, 512)
    got = ops.dequant("Q6_K", w, 24 * 2).cpu().numpy().reshape(24, 512)
    np.testing.assert_array_equal(got, full[16:40, 256:768])


@pytest.mark.parametrize("t,axis", [("Q8_0", 0), ("Q8_0", 1), ("Q4_K", 0), ("Q4_K", 1), ("Q6_K", 1)])
def test_shard_load_is_the_rank_slice(ops, oracle_mod, t, axis):
    """ef_weight_load_shard: rank r of 4 gets rows (axis 0) or columns (axis 1)
    [r * n/4, (r+1) * n/4) of the tensor, bit-exact; uneven splits are refused."""
    from elffuss_engine_b200._lib import EfError
    rows, k, n = 64, 2048, 4
    raw = formats.synth(t, rows, k, seed=12)
    full = oracle_mod.dequant(t, raw).reshape(rows, k)
    be, _ = formats.block_info(t)
    for r in range(n):
        w = ops.load_weight_shard(t, raw, rows, k, axis, r, n)
        nr, nk = (rows // n, k) if axis == 0 else (rows, k // n)
        got = ops.dequant(t, w, nr * nk // be).cpu().numpy().reshape(nr, nk)
        want = full[r * nr:(r + 1) * nr] if axis == 0 else full[:, r * nk:(r + 1) * nk]
        np.testing.assert_array_equal(got, want)
    with pytest.raises(EfError):
        ops.load_weight_shard(t, raw, rows, k, axis, 0, 3)   # 64 rows / 2048 columns do not split in 3


@pytest.mark.parametrize("t", ["Q8_0", "Q4_0", "Q2_K", "Q4_K", "Q5_K", "Q6_K", "IQ2_XXS", "IQ1_S"])
def test_gather_operator_rows_of_dequant(ops, t):
    """quant.gather (js/ops.js:1104-1118): the chosen rows of dequant(W), bit for
    bit, repeated ids included; an id past the table gives a zero row; a dim that
    is not a whole number of blocks is refused as the reference refuses it."""
    from elffuss_engine_b200._lib import EfError
    be, _ = formats.block_info(t)
    rows, k = 40, 512
    raw = formats.synth(t, rows, k, seed=9)
    w = ops.load_weight(t, raw, rows, k)
    wd = ops.dequant(t, w, rows * k // be).reshape(rows, k)
    ids = [3, 0, 39, 3, 40]
    out = ops.gather(t, w, ids, k, 5)
    assert out.shape == (5, k)
    assert torch.equal(out[:4], wd[[3, 0, 39, 3]])
    assert torch.equal(out[4], torch.zeros(k, device=out.device))
    with pytest.raises(EfError):
        ops.gather(t, w, ids, k + 16, 5)
