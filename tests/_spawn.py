"""Runs a test body as `world` spawned processes (one rank each) that meet
through a rendezvous file (no TCP port to collide with) and hands back what
each rank put on the queue; fails fast when a rank exits with an error."""
import os
import queue as _queue
import tempfile

import torch.multiprocessing as mp


def run_ranks(target, world, *args, timeout=300):
    """target(rank, world, init_method, q, *args) in each process; returns
    {rank: item[1:]} for the items (rank, ...) they put on q."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        init = "file://" + os.path.join(d, "rendezvous")
        procs = [ctx.Process(target=target, args=(r, world, init, q) + tuple(args)) for r in range(world)]
        for p in procs:
            p.start()
        got, waited = {}, 0.0
        try:
            while len(got) < world:
                try:
                    item = q.get(timeout=2.0)
                    got[item[0]] = item[1:]
                    continue
                except _queue.Empty:
                    waited += 2.0
                dead = [p for p in procs if p.exitcode not in (None, 0)]
                if dead:
                    raise AssertionError(f"rank process exited with {dead[0].exitcode}")
                if waited > timeout:
                    raise AssertionError("ranks did not finish in time")
            for p in procs:
                p.join(timeout=60)
                assert p.exitcode == 0
        finally:
            for p in procs:
                if p.is_alive():
                    p.kill()
                    p.join(timeout=10)
    return got
