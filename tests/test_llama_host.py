"""The Llama-shaped decoder's host side on the CPU: the Q4_K / Q6_K / Q8_0
quantizers against the CPU dequant, the config's byte counts, the shard rules
against slices of the whole tensors and a 2-rank gloo run of the CPU forward
on the shards against the unsharded forward."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import __graft_entry__  # noqa: E402  (spawned ranks import this module before conftest runs)

__graft_entry__.package()

import numpy as np  # noqa: E402
import pytest  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import oracle  # noqa: E402
from elffuss_engine_b200.llama import LlamaConfig, shard_weights, synth_weights  # noqa: E402
from elffuss_engine_b200.quantize import quantize  # noqa: E402
from oracle.llama_ref import LlamaOracle, rope_norm  # noqa: E402

from _spawn import run_ranks  # noqa: E402

MED = dict(hidden=512, layers=2, heads=8, kv_heads=4, head_dim=128, ffn=1024, vocab=1024, max_pos=64)


@pytest.mark.parametrize("t,step", [("Q4_K", 1 / 15), ("Q6_K", 1 / 32), ("Q8_0", 1 / 127)])
def test_quantizer_blocks_decode_to_the_tensor(t, step):
    g = torch.Generator().manual_seed(1)
    w = torch.empty(48, 1024).normal_(0, 0.02, generator=g)
    w[3, :256] = 0.0                                   # an all-zero superblock
    w[5, 256:512] = torch.linspace(-0.1, 0.1, 256)
    raw = quantize(t, w).numpy()
    deq = oracle.dequant(t, raw).reshape(48, 1024)
    assert np.all(deq[3, :256] == 0)
    # per 32-wide group: error within a few steps of the group's range
    x = w.numpy().reshape(48, -1, 32)
    err = np.abs(deq.reshape(48, -1, 32) - x).max(axis=2)
    rng = np.abs(x).max(axis=2)
    assert np.all(err <= 3 * step * 2 * rng + 1e-6)


def test_config4_bytes_per_token():
    c = LlamaConfig()
    assert c.step_weight_bytes() == 4_633_632_768
    assert c.weight_type("blk.0.ffn_down") == "Q6_K" and c.weight_type("blk.1.ffn_down") == "Q4_K"
    assert c.weight_type("blk.7.attn_v") == "Q6_K" and c.weight_type("output") == "Q6_K"
    assert c.weight_type("token_embd") == "Q4_K" and c.weight_type("blk.3.attn_q") == "Q4_K"


def test_rope_norm_pairs_adjacent_elements():
    x = np.random.default_rng(0).standard_normal((2, 8))
    y = rope_norm(x, 3, 1e4)
    th = 3 * 1e4 ** (-2.0 * np.arange(4) / 8)
    assert np.allclose(y[:, 0::2] ** 2 + y[:, 1::2] ** 2, x[:, 0::2] ** 2 + x[:, 1::2] ** 2)
    assert np.allclose(y[:, 2], x[:, 2] * np.cos(th[1]) - x[:, 3] * np.sin(th[1]))


def _deq(val):
    raw, rows, k, t = val
    return oracle.dequant(t, raw.numpy()).reshape(rows, k)


@pytest.mark.parametrize("world", [2, 4])
def test_shards_are_slices_of_the_whole(world):
    cfg = LlamaConfig(**MED)
    w = synth_weights(cfg, seed=2)
    D, F, V = cfg.head_dim, cfg.ffn, cfg.vocab
    Hl, KVl, Fl, Vl = cfg.heads // world, cfg.kv_heads // world, F // world, V // world
    full = {n: _deq(v) for n, v in w.items() if isinstance(v, tuple)}
    for r in range(world):
        s = shard_weights(cfg, w, r, world)
        assert np.array_equal(_deq(s["token_embd"]), full["token_embd"])
        assert np.array_equal(_deq(s["output"]), full["output"][r * Vl:(r + 1) * Vl])
        for l in range(cfg.layers):
            p = f"blk.{l}."
            assert np.array_equal(_deq(s[p + "attn_q"]), full[p + "attn_q"][r * Hl * D:(r + 1) * Hl * D])
            assert np.array_equal(_deq(s[p + "attn_k"]), full[p + "attn_k"][r * KVl * D:(r + 1) * KVl * D])
            assert np.array_equal(_deq(s[p + "attn_v"]), full[p + "attn_v"][r * KVl * D:(r + 1) * KVl * D])
            assert np.array_equal(_deq(s[p + "attn_output"]), full[p + "attn_output"][:, r * Hl * D:(r + 1) * Hl * D])
            assert np.array_equal(_deq(s[p + "ffn_gate"]), full[p + "ffn_gate"][r * Fl:(r + 1) * Fl])
            assert np.array_equal(_deq(s[p + "ffn_up"]), full[p + "ffn_up"][r * Fl:(r + 1) * Fl])
            assert np.array_equal(_deq(s[p + "ffn_down"]), full[p + "ffn_down"][:, r * Fl:(r + 1) * Fl])


def test_shard_rejects_slices_off_the_superblocks():
    cfg = LlamaConfig(**MED)
    with pytest.raises(ValueError):
        shard_weights(cfg, synth_weights(cfg, seed=2), 0, 8)     # ffn slice 128


def _np(w):
    return {k: ((v[0].numpy(), v[1], v[2], v[3]) if isinstance(v, tuple) else v.numpy()) for k, v in w.items()}


def _rank_main(rank, world, init, q, prefix, last, n):
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        cfg = LlamaConfig(**MED)
        w = shard_weights(cfg, synth_weights(cfg, seed=2), rank, world)

        def allreduce(v):
            t = torch.from_numpy(np.ascontiguousarray(v, np.float64))
            dist.all_reduce(t)
            return t.numpy()

        def allgather(pair):
            out = [None] * world
            dist.all_gather_object(out, pair)
            return out

        q.put((rank, LlamaOracle(cfg, _np(w), rank, world, allreduce, allgather).generate(prefix, last, n)))
    finally:
        dist.destroy_process_group()


def test_two_rank_forward_matches_unsharded():
    cfg = LlamaConfig(**MED)
    ids = np.random.default_rng(7).integers(0, cfg.vocab, 10)
    prefix, last, n = ids[:-1], int(ids[-1]), 6
    want = LlamaOracle(cfg, _np(synth_weights(cfg, seed=2))).generate(prefix, last, n)
    got = {r: v[0] for r, v in run_ranks(_rank_main, 2, prefix, last, n).items()}
    assert got[0] == want and got[1] == want
