"""The decoder-step kernels and the synthetic LFM3 decoder on the GPU, against
the CPU restatement (oracle/lfm3_ref.py): each operation on random data, then
greedy decoding at a reduced shape token for token."""
import ctypes

import numpy as np
import pytest
import torch

from elffuss_engine_b200 import formats
from elffuss_engine_b200._lib import check, lib
from elffuss_engine_b200.lfm3 import SMALL, LFM3Config, LFM3Decoder, synth_weights
from oracle.lfm3_ref import LFM3Oracle, dequant_q8_0, rmsnorm, rope_neox

pytestmark = pytest.mark.gpu


def P(t):
    return ctypes.c_void_p(t.data_ptr())


def _np_weights(w):
    return {k: ((v[0].numpy(), v[1], v[2]) if isinstance(v, tuple) else v.numpy()) for k, v in w.items()}


def test_rmsnorm_and_norm_add_norm(ops):
    L, h = lib(), ops.ctx.bind()
    g = torch.Generator("cuda").manual_seed(1)
    x = torch.randn(3, 2048, device="cuda", generator=g)
    w = torch.rand(2048, device="cuda", generator=g) + 0.5
    y = torch.empty_like(x)
    check(L.ef_rmsnorm(h, P(x), P(w), 3, 2048, ctypes.c_float(1e-5), P(y)), h)
    ref = rmsnorm(x.double().cpu().numpy(), w.double().cpu().numpy(), 1e-5)
    assert np.allclose(y.cpu().numpy(), ref, rtol=2e-5, atol=2e-6)
    o = torch.randn(3, 2048, device="cuda", generator=g)
    w2 = torch.rand(2048, device="cuda", generator=g) + 0.5
    xr = x.clone()
    nrm = torch.empty_like(x)
    check(L.ef_norm_add_norm(h, P(o), P(w), P(xr), P(w2), 3, 2048, ctypes.c_float(1e-5), P(nrm)), h)
    xn = x.double().cpu().numpy() + rmsnorm(o.double().cpu().numpy(), w.double().cpu().numpy(), 1e-5)
    assert np.allclose(xr.cpu().numpy(), xn, rtol=2e-5, atol=2e-5)
    assert np.allclose(nrm.cpu().numpy(), rmsnorm(xn, w2.double().cpu().numpy(), 1e-5), rtol=5e-5, atol=5e-5)


def test_shortconv_tokens_and_state(ops):
    L, h = lib(), ops.ctx.bind()
    C, T = 300, 5
    g = torch.Generator("cuda").manual_seed(2)
    bcx = torch.randn(T, 3 * C, device="cuda", generator=g)
    w = torch.randn(C, 3, device="cuda", generator=g)
    st0 = torch.randn(2, C, device="cuda", generator=g)
    st = st0.clone()
    y = torch.empty(T, C, device="cuda")
    check(L.ef_shortconv(h, P(bcx), P(w), P(st), T, C, 3, P(y)), h)
    b, c, xs = [a.double().cpu().numpy() for a in (bcx[:, :C], bcx[:, C:2 * C], bcx[:, 2 * C:])]
    win = np.concatenate([st0.double().cpu().numpy(), b * xs], axis=0)   # [2 + T][C]
    wn = w.double().cpu().numpy()
    ref = np.stack([c[t] * np.sum(win[t:t + 3].T * wn, axis=1) for t in range(T)])
    assert np.allclose(y.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)
    assert np.allclose(st.cpu().numpy(), win[-2:], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("window", [0, 5])
def test_qk_rope_cache_and_attention(ops, window):
    L, h = lib(), ops.ctx.bind()
    H, KV, D, maxp, pos = 8, 2, 64, 32, 11
    g = torch.Generator("cuda").manual_seed(3)
    kc = torch.randn(maxp, KV, D, device="cuda", generator=g)
    vc = torch.randn(maxp, KV, D, device="cuda", generator=g)
    q = torch.randn(H * D, device="cuda", generator=g)
    k = torch.randn(KV * D, device="cuda", generator=g)
    v = torch.randn(KV * D, device="cuda", generator=g)
    wq = torch.rand(D, device="cuda", generator=g) + 0.5
    wk = torch.rand(D, device="cuda", generator=g) + 0.5
    gate = torch.randn(H, device="cuda", generator=g)
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    q0, kc0 = q.double().cpu().numpy(), kc.double().cpu().numpy()
    check(L.ef_qk_norm_rope_cache(h, P(q), P(k), P(v), P(wq), P(wk), P(p), maxp, H, KV, D, ctypes.c_float(1e6),
                                  ctypes.c_float(1e-5), P(kc), P(vc)), h)
    qr = rope_neox(rmsnorm(q0.reshape(H, D), wq.double().cpu().numpy(), 1e-5), pos, 1e6)
    kr = rope_neox(rmsnorm(k.double().cpu().numpy().reshape(KV, D), wk.double().cpu().numpy(), 1e-5), pos, 1e6)
    assert np.allclose(q.cpu().numpy().reshape(H, D), qr, rtol=1e-4, atol=1e-4)
    assert np.allclose(kc[pos].cpu().numpy(), kr, rtol=1e-4, atol=1e-4)
    assert np.allclose(vc[pos].cpu().numpy(), v.cpu().numpy().reshape(KV, D))
    assert np.allclose(kc[pos + 1].cpu().numpy(), kc0[pos + 1])          # nothing else written
    out = torch.empty(H * D, device="cuda")
    check(L.ef_attn_decode(h, P(q), P(kc), P(vc), P(gate), P(p), maxp, window, H, KV, D, P(out)), h)
    K, V, Q = kc.double().cpu().numpy(), vc.double().cpu().numpy(), q.double().cpu().numpy().reshape(H, D)
    keys = np.arange(pos + 1)
    vis = (window == 0) | (pos - keys < window)
    ref = np.empty((H, D))
    for hh in range(H):
        kv = hh // (H // KV)
        s = np.where(vis, K[:pos + 1, kv] @ Q[hh] / 8.0, -np.inf)
        e = np.exp(s - s.max())
        ref[hh] = (e / e.sum()) @ V[:pos + 1, kv] / (1 + np.exp(-gate[hh].item()))
    assert np.allclose(out.cpu().numpy().reshape(H, D), ref, rtol=1e-4, atol=1e-5)


def test_argmax_step_lowest_index_wins_ties(ops):
    L, h = lib(), ops.ctx.bind()
    logits = torch.randn(65536, device="cuda", generator=torch.Generator("cuda").manual_seed(4))
    m = logits.max().item()
    logits[40000] = m + 1.0
    logits[7] = m + 1.0
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos = torch.tensor([4], dtype=torch.int32, device="cuda")
    outt = torch.full((8,), -1, dtype=torch.int32, device="cuda")
    check(L.ef_argmax_step(h, P(logits), 65536, P(tok), P(pos), P(outt), 3, 8), h)
    assert tok.item() == 7 and pos.item() == 5 and outt[2].item() == 7


def test_gather_rows_are_exact_dequant(ops):
    L, h = lib(), ops.ctx.bind()
    rows, k = 100, 256
    raw = formats.quantize_q8_0(np.random.default_rng(6).standard_normal((rows, k)).astype(np.float32) * 0.02)
    w = ops.load_weight("Q8_0", raw, rows, k)
    ids = torch.tensor([5, 99, 0, 77, 200], dtype=torch.int32, device="cuda")
    out = torch.empty(5, k, device="cuda")
    check(L.ef_gather(h, w.h, P(ids), 5, P(out)), h)
    ref = dequant_q8_0(raw, rows, k)
    got = out.cpu().numpy()
    for i, r in enumerate([5, 99, 0, 77]):
        assert np.array_equal(got[i], ref[r])
    assert np.all(got[4] == 0)                                   # id outside the rows


@pytest.mark.parametrize("t", ["Q8_0", "Q4_K", "Q6_K"])
def test_gather_rmsnorm_equals_gather_then_norm(ops, t):
    L, h = lib(), ops.ctx.bind()
    rows, k = 50, 1024
    raw = formats.synth(t, rows, k, seed=3)
    w = ops.load_weight(t, raw, rows, k)
    ids = torch.tensor([4, 49, 0, 60], dtype=torch.int32, device="cuda")
    wn = torch.rand(k, device="cuda") + 0.5
    x, nrm = torch.empty(4, k, device="cuda"), torch.empty(4, k, device="cuda")
    check(L.ef_gather_rmsnorm(h, w.h, P(ids), 4, P(wn), ctypes.c_float(1e-5), P(x), P(nrm)), h)
    xg = torch.empty(4, k, device="cuda")
    check(L.ef_gather(h, w.h, P(ids), 4, P(xg)), h)
    assert torch.equal(x, xg)                                   # the same bits as the gather
    ref = rmsnorm(xg.double().cpu().numpy(), wn.double().cpu().numpy(), 1e-5)
    assert np.allclose(nrm.cpu().numpy()[:3], ref[:3], rtol=2e-5, atol=2e-6)
    assert torch.all(nrm[3] == 0)


def test_small_decoder_greedy_tokens_match_oracle(ops):
    cfg = LFM3Config(**SMALL)
    w = synth_weights(cfg, seed=1)
    prompt = torch.tensor(np.random.default_rng(5).integers(0, cfg.vocab, 20), dtype=torch.int32)
    want = LFM3Oracle(cfg, _np_weights(w)).generate(prompt.numpy(), 32)
    dec = LFM3Decoder(ops, cfg, w)
    got_graph = dec.generate(prompt, 32, use_graph=True)
    got_eager = dec.generate(prompt, 32, use_graph=False)
    got_steps = dec.generate(prompt, 32, use_graph=True, batched_prompt=False)
    assert got_graph == got_eager
    assert got_graph == want
    assert got_steps == want
