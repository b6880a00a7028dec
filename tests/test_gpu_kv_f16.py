"""f16 KV caches (the reference's kvF16 option, js/model.js:906-946,
js/kernels.attn.wgsl.js:51-55) on the GPU: the cache write stores exactly the
f32 path's k (after norm and RoPE) and v rounded to f16, to nearest even, and
leaves q as the f32 path leaves it. Attention reading f16 caches: the tiled
prompt kernel, the one-CTA-per-row kernel and the decode split for 8 query
heads per cache head give the same bits as the f32 kernels reading f32 caches
that hold the same f16 values; the decode split for up to 4 query heads per
cache head runs on the tensor cores (q and the probabilities split into two
f16 parts) and agrees with them to 2e-5 of the output's magnitude."""
import ctypes

import pytest
import torch

from elffuss_engine_b200._lib import check, lib

pytestmark = pytest.mark.gpu


def P(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


@pytest.mark.parametrize("D,mode,norm", [(128, 0, False), (64, 2, True), (128, 2, True)])
def test_cache_write_is_the_f32_write_rounded(ops, D, mode, norm):
    L, h = lib(), ops.ctx.bind()
    S, T, H, KV, maxp = 2, 5, 8, 2, 40
    g = torch.Generator("cuda").manual_seed(D + mode)
    q = torch.randn(S * T, H * D, device="cuda", generator=g)
    k = torch.randn(S * T, KV * D, device="cuda", generator=g) * 3
    v = torch.randn(S * T, KV * D, device="cuda", generator=g) * 3
    wq = torch.rand(D, device="cuda", generator=g) + 0.5 if norm else None
    wk = torch.rand(D, device="cuda", generator=g) + 0.5 if norm else None
    pd = torch.tensor([3, 34], dtype=torch.int32, device="cuda")   # the second runs past the caches
    kc32 = torch.zeros(S, maxp, KV, D, device="cuda")
    vc32 = torch.zeros_like(kc32)
    kc16 = torch.full((S, maxp, KV, D), 7.0, dtype=torch.float16, device="cuda")   # untouched rows stay 7
    vc16 = kc16.clone()
    q32, q16 = q.clone(), q.clone()
    args = (P(pd), S, T, maxp, H, KV, D, mode, ctypes.c_float(1e4), ctypes.c_float(1e-5))
    check(L.ef_rope_cache(h, P(q32), P(k), P(v), P(wq), P(wk), *args, P(kc32), P(vc32)), h)
    check(L.ef_rope_cache_f16(h, P(q16), P(k), P(v), P(wq), P(wk), *args, P(kc16), P(vc16)), h)
    torch.cuda.synchronize()
    assert torch.equal(q32, q16)
    written = torch.zeros(S, maxp, dtype=torch.bool)
    for s, p0 in enumerate([3, 34]):
        for t in range(T):
            if p0 + t < maxp:
                written[s, p0 + t] = True
    wm = written.cuda()
    assert torch.equal(kc16[wm], kc32[wm].half())
    assert torch.equal(vc16[wm], vc32[wm].half())
    assert bool((kc16[~wm] == 7).all()) and bool((vc16[~wm] == 7).all())


# (D, H, KV, S, T, pos, window, gated): T = 1 with G in {1, 2, 4, 8} is the
# decode split over the keys, T > 1 the tiled prompt kernel, G = 3 the
# one-CTA-per-row kernel
CASES = [
    (128, 8, 8, 3, 1, [0, 17, 300], 0, False),
    (128, 32, 8, 2, 1, [4095, 1000], 0, False),
    (64, 16, 2, 1, 1, [700], 64, True),
    (64, 32, 8, 1, 1, [5000], 4096, True),
    (128, 8, 2, 2, 37, [0, 100], 0, False),
    (64, 8, 2, 1, 200, [30], 50, True),
    (128, 6, 2, 2, 3, [5, 60], 0, True),
    (128, 4, 2, 3, 1, [3, 40, 1000], 0, True),
    (64, 8, 2, 2, 1, [17, 4000], 100, False),
]


@pytest.mark.parametrize("D,H,KV,S,T,pos,window,gated", CASES)
def test_attention_on_f16_caches_equals_f32_kernels(ops, D, H, KV, S, T, pos, window, gated):
    L, h = lib(), ops.ctx.bind()
    maxp = max(pos) + T + 8
    g = torch.Generator("cuda").manual_seed(D * 7 + H + T)
    kc16 = (torch.randn(S, maxp, KV, D, device="cuda", generator=g) * 2).half()
    vc16 = (torch.randn(S, maxp, KV, D, device="cuda", generator=g) * 2).half()
    kc32, vc32 = kc16.float(), vc16.float()
    q = torch.randn(S * T, H * D, device="cuda", generator=g)
    gate = torch.randn(S * T, H, device="cuda", generator=g) if gated else None
    pd = torch.tensor(pos, dtype=torch.int32, device="cuda")
    o32 = torch.empty(S * T, H * D, device="cuda")
    o16 = torch.empty_like(o32)
    check(L.ef_attention(h, P(q), P(kc32), P(vc32), P(gate), P(pd), S, T, maxp, window, H, KV, D, P(o32)), h)
    check(L.ef_attention_f16(h, P(q), P(kc16), P(vc16), P(gate), P(pd), S, T, maxp, window, H, KV, D, P(o16)), h)
    torch.cuda.synchronize()
    assert torch.isfinite(o32).all()
    _agree(o32, o16, T == 1 and H // KV <= 4)


def _agree(o32, o16, mma):
    if mma:       # tensor-core decode split: f16 operands, q and p split in two
        assert torch.isfinite(o16).all()
        assert float((o16 - o32).abs().max()) <= 2e-5 * float(o32.abs().max())
    else:
        assert torch.equal(o32, o16)


def test_decode_entry_on_f16_caches(ops):
    L, h = lib(), ops.ctx.bind()
    D, H, KV, maxp, window = 64, 32, 8, 5120, 4096
    g = torch.Generator("cuda").manual_seed(3)
    kc16 = torch.randn(maxp, KV, D, device="cuda", generator=g).half()
    vc16 = torch.randn(maxp, KV, D, device="cuda", generator=g).half()
    q = torch.randn(H * D, device="cuda", generator=g)
    gate = torch.randn(H, device="cuda", generator=g)
    pd = torch.tensor([4500], dtype=torch.int32, device="cuda")
    o32 = torch.empty(H * D, device="cuda")
    o16 = torch.empty_like(o32)
    kc32, vc32 = kc16.float(), vc16.float()
    check(L.ef_attn_decode(h, P(q), P(kc32), P(vc32), P(gate), P(pd), maxp, window, H, KV, D, P(o32)), h)
    check(L.ef_attn_decode_f16(h, P(q), P(kc16), P(vc16), P(gate), P(pd), maxp, window, H, KV, D, P(o16)), h)
    torch.cuda.synchronize()
    _agree(o32, o16, True)
