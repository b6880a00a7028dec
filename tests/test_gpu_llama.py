"""The batched attention kernels and the Llama-shaped decoder on the GPU,
against numpy and the CPU restatement (oracle/llama_ref.py): RoPE (NORM and
NEOX pairing, head_dim 64 and 128) with the cache write for several sequences
of several tokens, causal attention over those caches, SwiGLU, per-row argmax;
then greedy decoding of 3 sequences of a reduced-shape model (prompt through
the GEMM path, steps through the GEMV path), token for token, on 1 GPU and
tensor-parallel on 2 (skipped with fewer)."""
import ctypes
import datetime
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import __graft_entry__  # noqa: E402  (spawned ranks import this module before conftest runs)

__graft_entry__.package()

import numpy as np  # noqa: E402
import pytest  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from elffuss_engine_b200._lib import check, lib  # noqa: E402
from elffuss_engine_b200.llama import SMALL, LlamaConfig, LlamaDecoder, shard_weights, synth_weights  # noqa: E402
from oracle.lfm3_ref import rmsnorm, rope_neox  # noqa: E402
from oracle.llama_ref import LlamaOracle, rope_norm  # noqa: E402

from _spawn import run_ranks  # noqa: E402

pytestmark = pytest.mark.gpu
MED = dict(hidden=512, layers=2, heads=8, kv_heads=4, head_dim=128, ffn=1024, vocab=1024, max_pos=64)


def P(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _np(w):
    return {k: ((v[0].numpy(), v[1], v[2], v[3]) if isinstance(v, tuple) else v.numpy()) for k, v in w.items()}


@pytest.mark.parametrize("D,mode,norm", [(128, 0, False), (64, 2, True), (128, 2, False), (64, 0, True)])
def test_rope_cache_and_attention_batched(ops, D, mode, norm):
    L, h = lib(), ops.ctx.bind()
    S, T, H, KV, maxp = 2, 3, 4, 2, 24
    pos = [5, 9]
    g = torch.Generator("cuda").manual_seed(D + mode)
    kc = torch.randn(S, maxp, KV, D, device="cuda", generator=g)
    vc = torch.randn(S, maxp, KV, D, device="cuda", generator=g)
    q = torch.randn(S * T, H * D, device="cuda", generator=g)
    k = torch.randn(S * T, KV * D, device="cuda", generator=g)
    v = torch.randn(S * T, KV * D, device="cuda", generator=g)
    wq = torch.rand(D, device="cuda", generator=g) + 0.5 if norm else None
    wk = torch.rand(D, device="cuda", generator=g) + 0.5 if norm else None
    pd = torch.tensor(pos, dtype=torch.int32, device="cuda")
    q0, k0, kc0 = q.double().cpu().numpy(), k.double().cpu().numpy(), kc.double().cpu().numpy()
    check(L.ef_rope_cache(h, P(q), P(k), P(v), P(wq), P(wk), P(pd), S, T, maxp, H, KV, D, mode,
                          ctypes.c_float(1e4), ctypes.c_float(1e-5), P(kc), P(vc)), h)
    rot = rope_neox if mode == 2 else rope_norm
    K, V = kc.double().cpu().numpy(), vc.double().cpu().numpy()
    for s in range(S):
        for t in range(T):
            r, p = s * T + t, pos[s] + t
            qn, kn = q0[r].reshape(H, D), k0[r].reshape(KV, D)
            if norm:
                qn = rmsnorm(qn, wq.double().cpu().numpy(), 1e-5)
                kn = rmsnorm(kn, wk.double().cpu().numpy(), 1e-5)
            assert np.allclose(q[r].cpu().numpy().reshape(H, D), rot(qn, p, 1e4), rtol=1e-4, atol=1e-4)
            assert np.allclose(K[s, p], rot(kn, p, 1e4), rtol=1e-4, atol=1e-4)
            assert np.array_equal(vc[s, p].cpu().numpy(), v[r].cpu().numpy().reshape(KV, D))
        assert np.array_equal(K[s, pos[s] + T:], kc0[s, pos[s] + T:])        # nothing else written
    for window in (0, 4):
        out = torch.empty(S * T, H * D, device="cuda")
        gate = torch.randn(S * T, H, device="cuda", generator=g)
        check(L.ef_attention(h, P(q), P(kc), P(vc), P(gate), P(pd), S, T, maxp, window, H, KV, D, P(out)), h)
        Q = q.double().cpu().numpy()
        for s in range(S):
            for t in range(T):
                r, p = s * T + t, pos[s] + t
                keys = np.arange(p + 1)
                vis = (window == 0) | (p - keys < window)
                for hh in range(H):
                    kv = hh // (H // KV)
                    sc = np.where(vis, K[s, :p + 1, kv] @ Q[r].reshape(H, D)[hh] / np.sqrt(D), -np.inf)
                    e = np.exp(sc - sc.max())
                    want = (e / e.sum()) @ V[s, :p + 1, kv] / (1 + np.exp(-gate[r, hh].item()))
                    assert np.allclose(out[r].cpu().numpy().reshape(H, D)[hh], want, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("D,H,KV,S,T,pos,window,gated", [
    (128, 32, 8, 1, 700, [0], 0, False),          # the 8B shape, G = 4
    (64, 16, 2, 2, 300, [0, 50], 100, True),      # G = 8, a window, two sequences at different offsets
    (128, 8, 8, 1, 257, [3], 0, True),            # G = 1
    (64, 8, 4, 2, 130, [10, 0], 0, False),        # G = 2
    (128, 16, 2, 1, 9, [0], 3, False),            # a short prompt, window smaller than a key tile
])
def test_prompt_attention_tiled(ops, D, H, KV, S, T, pos, window, gated):
    """Several new tokens per sequence (the prompt path): key tiles shared by a
    block of queries with an online softmax, against float64."""
    L, h = lib(), ops.ctx.bind()
    maxp = max(pos) + T + 5
    g = torch.Generator("cuda").manual_seed(D + H + T)
    kc = torch.randn(S, maxp, KV, D, device="cuda", generator=g)
    vc = torch.randn(S, maxp, KV, D, device="cuda", generator=g)
    q = torch.randn(S * T, H * D, device="cuda", generator=g) * 2
    gate = torch.randn(S * T, H, device="cuda", generator=g) if gated else None
    pd = torch.tensor(pos, dtype=torch.int32, device="cuda")
    out = torch.empty(S * T, H * D, device="cuda")
    check(L.ef_attention(h, P(q), P(kc), P(vc), P(gate), P(pd), S, T, maxp, window, H, KV, D, P(out)), h)
    G = H // KV
    for s in range(S):
        Q = q[s * T:(s + 1) * T].double().reshape(T, H, D)
        K = kc[s].double().repeat_interleave(G, dim=1)          # [maxp][H][D]
        V = vc[s].double().repeat_interleave(G, dim=1)
        sc = torch.einsum("thd,khd->htk", Q, K) / D ** 0.5
        qp = torch.arange(T, device="cuda")[:, None] + pos[s]
        key = torch.arange(maxp, device="cuda")[None, :]
        vis = (key <= qp) & ((window == 0) | (qp - key < window))
        sc = sc.masked_fill(~vis[None], float("-inf"))
        want = torch.einsum("htk,khd->thd", torch.softmax(sc, dim=-1), V)
        if gated:
            want = want * torch.sigmoid(gate[s * T:(s + 1) * T].double())[:, :, None]
        got = out[s * T:(s + 1) * T].double().reshape(T, H, D)
        assert torch.allclose(got, want, rtol=1e-4, atol=1e-5), float((got - want).abs().max())


@pytest.mark.parametrize("D,H,KV", [(128, 8, 2), (64, 32, 8), (128, 4, 4), (64, 16, 2)])
def test_decode_attention_split_over_long_caches(ops, D, H, KV):
    """One new token per sequence: the keys split in ranges of 256 over CTAs,
    then merged; sequences at different depths, with and without a window."""
    L, h = lib(), ops.ctx.bind()
    S, maxp, pos = 3, 1200, [1000, 700, 5]
    g = torch.Generator("cuda").manual_seed(D + H)
    kc = torch.randn(S, maxp, KV, D, device="cuda", generator=g)
    vc = torch.randn(S, maxp, KV, D, device="cuda", generator=g)
    q = torch.randn(S, H * D, device="cuda", generator=g) * 2
    pd = torch.tensor(pos, dtype=torch.int32, device="cuda")
    K, V, Q = kc.double().cpu().numpy(), vc.double().cpu().numpy(), q.double().cpu().numpy()
    for window in (0, 300):
        gate = torch.randn(S, H, device="cuda", generator=g) if window else None
        out = torch.empty(S, H * D, device="cuda")
        check(L.ef_attention(h, P(q), P(kc), P(vc), P(gate), P(pd), S, 1, maxp, window, H, KV, D, P(out)), h)
        for s in range(S):
            p = pos[s]
            keys = np.arange(p + 1)
            vis = (window == 0) | (p - keys < window)
            for hh in range(H):
                kv = hh // (H // KV)
                sc = np.where(vis, K[s, :p + 1, kv] @ Q[s].reshape(H, D)[hh] / np.sqrt(D), -np.inf)
                e = np.exp(sc - sc.max())
                want = (e / e.sum()) @ V[s, :p + 1, kv]
                if gate is not None:
                    want = want / (1 + np.exp(-gate[s, hh].item()))
                assert np.allclose(out[s].cpu().numpy().reshape(H, D)[hh], want, rtol=1e-4, atol=1e-5)


def test_swiglu_and_argmax_rows(ops):
    L, h = lib(), ops.ctx.bind()
    g = torch.Generator("cuda").manual_seed(9)
    a, b = torch.randn(3000, device="cuda", generator=g), torch.randn(3000, device="cuda", generator=g)
    out = torch.empty(3000, device="cuda")
    check(L.ef_swiglu(h, P(a), P(b), 3000, P(out)), h)
    an, bn = a.double().cpu().numpy(), b.double().cpu().numpy()
    assert np.allclose(out.cpu().numpy(), an / (1 + np.exp(-an)) * bn, rtol=1e-5, atol=1e-6)
    lg = torch.randn(3, 5000, device="cuda", generator=g)
    lg[1, 17] = lg[1, 4000] = 50.0                       # tie: the lower index wins
    tok = torch.zeros(3, dtype=torch.int32, device="cuda")
    pos = torch.tensor([2, 7, 0], dtype=torch.int32, device="cuda")
    outt = torch.full((3, 4), -1, dtype=torch.int32, device="cuda")
    check(L.ef_argmax_rows(h, P(lg), 3, 5000, P(tok), P(pos), P(outt), 1, 4), h)
    want = lg.argmax(dim=1).cpu().tolist()
    want[1] = 17
    assert tok.cpu().tolist() == want and pos.cpu().tolist() == [3, 8, 1]
    assert outt[0, 2].item() == want[0] and outt[2, 0].item() == want[2] and outt[1].tolist() == [-1] * 4


def _run_small(ops, cfg, w, prefix, lasts, n, rank=0, world=1, comm=None):
    dec = LlamaDecoder(ops, cfg, w, batch=len(lasts), rank=rank, world=world, comm=comm)
    prompt = torch.tensor(list(prefix) + [int(lasts[0])], dtype=torch.int32)
    got_graph = dec.generate(prompt, lasts, n, use_graph=True)
    got_eager = dec.generate(prompt, lasts, n, use_graph=False)
    dec.graph = None
    return got_graph, got_eager


def test_small_llama_three_sequences_match_oracle(ops):
    cfg = LlamaConfig(**SMALL)
    w = synth_weights(cfg, seed=3)
    ids = np.random.default_rng(4).integers(0, cfg.vocab, 26)
    prefix, lasts, n = ids[:23], [int(t) for t in ids[23:]], 16
    orc = LlamaOracle(cfg, _np(w))
    want = [orc.generate(prefix, last, n) for last in lasts]
    got_graph, got_eager = _run_small(ops, cfg, w, prefix, lasts, n)
    assert got_graph == got_eager
    assert got_graph == want


def _rank_main(rank, world, init, q, prefix, lasts, n, use_comm):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=init, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        from elffuss_engine_b200.ops import QuantOps
        from elffuss_engine_b200.tp import TPComm
        cfg = LlamaConfig(**MED)
        w = shard_weights(cfg, synth_weights(cfg, seed=2), rank, world)
        ops = QuantOps(rank)
        comm = TPComm(ops, rank, world) if use_comm else None
        q.put((rank,) + _run_small(ops, cfg, w, prefix, lasts, n, rank, world, comm))
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("use_comm", [False, True], ids=["nccl", "peer"])
def test_two_gpu_tensor_parallel_llama_matches_oracle(use_comm):
    cfg = LlamaConfig(**MED)
    ids = np.random.default_rng(8).integers(0, cfg.vocab, 14)
    prefix, lasts, n = ids[:12], [int(t) for t in ids[12:]], 12
    orc = LlamaOracle(cfg, _np(synth_weights(cfg, seed=2)))
    want = [orc.generate(prefix, last, n) for last in lasts]
    got = run_ranks(_rank_main, 2, prefix, lasts, n, use_comm)
    for r in range(2):
        assert got[r][0] == got[r][1] == want
