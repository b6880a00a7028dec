"""Tensor-parallel sharding of the LFM3 decoder, on the CPU: the shard rules
(lfm3.shard_weights) against slices of the whole tensors, and a 2-rank gloo
run of the CPU forward on the shards against the unsharded forward."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import __graft_entry__  # noqa: E402  (spawned ranks import this module before conftest runs)

__graft_entry__.package()

import numpy as np  # noqa: E402
import pytest  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from elffuss_engine_b200.lfm3 import SMALL, LFM3Config, shard_weights, synth_weights  # noqa: E402
from oracle.lfm3_ref import LFM3Oracle, dequant_q8_0  # noqa: E402

from _spawn import run_ranks  # noqa: E402

MEDIUM = dict(hidden=512, layers=3, attn_layers=(1,), heads=8, kv_heads=8, head_dim=64, ffn=1024, vocab=2048,
              window=8, max_pos=64)


def _np(w):
    return {k: ((v[0].numpy(), v[1], v[2]) if isinstance(v, tuple) else v.numpy()) for k, v in w.items()}


def _deq(val):
    raw, rows, k = val
    return dequant_q8_0(raw.numpy(), rows, k)


@pytest.mark.parametrize("world", [2, 8])
def test_shards_are_slices_of_the_whole(world):
    cfg = LFM3Config(**MEDIUM)
    w = synth_weights(cfg, seed=3)
    E, D, F, V = cfg.hidden, cfg.head_dim, cfg.ffn, cfg.vocab
    Hl, KVl, Ec, Fl, Vl = cfg.heads // world, cfg.kv_heads // world, E // world, F // world, V // world
    full = {n: _deq(v) for n, v in w.items() if isinstance(v, tuple)}
    for r in range(world):
        s = shard_weights(cfg, w, r, world)
        assert np.array_equal(_deq(s["token_embd"]), full["token_embd"])
        assert np.array_equal(_deq(s["output"]), full["token_embd"][r * Vl:(r + 1) * Vl])
        p = "blk.1."
        assert np.array_equal(_deq(s[p + "attn_q"]), full[p + "attn_q"][r * Hl * D:(r + 1) * Hl * D])
        assert np.array_equal(_deq(s[p + "attn_k"]), full[p + "attn_k"][r * KVl * D:(r + 1) * KVl * D])
        assert np.array_equal(_deq(s[p + "attn_v"]), full[p + "attn_v"][r * KVl * D:(r + 1) * KVl * D])
        assert np.array_equal(_deq(s[p + "attn_gate"]), full[p + "attn_gate"][r * Hl:(r + 1) * Hl])
        assert np.array_equal(_deq(s[p + "attn_output"]), full[p + "attn_output"][:, r * Hl * D:(r + 1) * Hl * D])
        p = "blk.0."
        inp = full[p + "shortconv.in_proj"]
        want = np.concatenate([inp[j * E + r * Ec:j * E + (r + 1) * Ec] for j in range(3)])
        assert np.array_equal(_deq(s[p + "shortconv.in_proj"]), want)
        assert torch.equal(s[p + "shortconv.conv"], w[p + "shortconv.conv"][r * Ec:(r + 1) * Ec])
        assert np.array_equal(_deq(s[p + "shortconv.out_proj"]), full[p + "shortconv.out_proj"][:, r * Ec:(r + 1) * Ec])
        for l in range(cfg.layers):
            p = f"blk.{l}."
            assert np.array_equal(_deq(s[p + "ffn_gate"]), full[p + "ffn_gate"][r * Fl:(r + 1) * Fl])
            assert np.array_equal(_deq(s[p + "ffn_up"]), full[p + "ffn_up"][r * Fl:(r + 1) * Fl])
            assert np.array_equal(_deq(s[p + "ffn_down"]), full[p + "ffn_down"][:, r * Fl:(r + 1) * Fl])
            assert torch.equal(s[p + "ffn_norm"], w[p + "ffn_norm"])


def test_shard_rejects_a_split_that_does_not_divide():
    cfg = LFM3Config(**SMALL)          # 2 KV heads
    with pytest.raises(ValueError):
        shard_weights(cfg, synth_weights(cfg, seed=1), 0, 4)


def _rank_main(rank, world, init, q, prompt, n):
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        cfg = LFM3Config(**SMALL)
        w = shard_weights(cfg, synth_weights(cfg, seed=1), rank, world)

        def allreduce(v):
            t = torch.from_numpy(np.ascontiguousarray(v, np.float64))
            dist.all_reduce(t)
            return t.numpy()

        def allgather(pair):
            out = [None] * world
            dist.all_gather_object(out, pair)
            return out

        toks = LFM3Oracle(cfg, _np(w), rank, world, allreduce, allgather).generate(prompt, n)
        q.put((rank, toks))
    finally:
        dist.destroy_process_group()


def test_two_rank_forward_matches_unsharded():
    cfg = LFM3Config(**SMALL)
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, 12)
    n = 10
    want = LFM3Oracle(cfg, _np(synth_weights(cfg, seed=1))).generate(prompt, n)
    got = {r: v[0] for r, v in run_ranks(_rank_main, 2, prompt, n).items()}
    assert got[0] == want and got[1] == want
