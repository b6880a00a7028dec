"""Tensor-parallel LFM3 decoding on 2 GPUs (skipped with fewer), with the
collectives through NCCL and through the library's peer-memory kernels
(tp.TPComm): each rank runs its shard (lfm3.shard_weights) with the
all-reduces and the sharded argmax captured in the step's CUDA graph; the
greedy tokens must be those of the unsharded CPU forward
(oracle/lfm3_ref.py)."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import __graft_entry__  # noqa: E402  (spawned ranks import this module before conftest runs)

__graft_entry__.package()

import datetime  # noqa: E402

import numpy as np  # noqa: E402
import pytest  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from elffuss_engine_b200.lfm3 import SMALL, LFM3Config, LFM3Decoder, shard_weights, synth_weights  # noqa: E402
from oracle.lfm3_ref import LFM3Oracle  # noqa: E402

from _spawn import run_ranks  # noqa: E402

pytestmark = pytest.mark.gpu


def _np(w):
    return {k: ((v[0].numpy(), v[1], v[2]) if isinstance(v, tuple) else v.numpy()) for k, v in w.items()}


def _rank_main(rank, world, init, q, prompt, n, use_comm):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=init, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    dec = None
    try:
        from elffuss_engine_b200.ops import QuantOps
        ops = QuantOps(rank)
        cfg = LFM3Config(**SMALL)
        comm = None
        if use_comm:
            from elffuss_engine_b200.tp import TPComm
            comm = TPComm(ops, rank, world)
        dec = LFM3Decoder(ops, cfg, shard_weights(cfg, synth_weights(cfg, seed=1), rank, world), rank, world,
                          comm=comm)
        pt = torch.tensor(prompt, dtype=torch.int32)
        got_graph = dec.generate(pt, n, use_graph=True)
        got_eager = dec.generate(pt, n, use_graph=False)
        q.put((rank, got_graph, got_eager))
    finally:
        if dec is not None:
            dec.graph = None          # the graph holds NCCL work: release it before the group
        torch.cuda.synchronize()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("use_comm", [False, True], ids=["nccl", "peer"])
def test_two_gpu_tensor_parallel_tokens_match_oracle(use_comm):
    cfg = LFM3Config(**SMALL)
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, 20)
    n = 32
    want = LFM3Oracle(cfg, _np(synth_weights(cfg, seed=1))).generate(prompt, n)
    got = run_ranks(_rank_main, 2, prompt, n, use_comm)
    for r in range(2):
        assert got[r][0] == got[r][1]
        assert got[r][0] == want
