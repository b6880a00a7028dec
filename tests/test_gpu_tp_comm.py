"""The peer-memory collectives (ef_tp_*, tp.TPComm) on 2 GPUs (skipped with
fewer): the all-reduce is the rank-order sum bit for bit on every rank, the
all-gather concatenates in rank order, both replay correctly from a CUDA
graph; a rank that never arrives makes the other's wait run out, which is
reported as EF_ERR_TIMEOUT with the context still usable."""
import datetime
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import __graft_entry__  # noqa: E402  (spawned ranks import this module before conftest runs)

__graft_entry__.package()

import pytest  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from _spawn import run_ranks  # noqa: E402

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]


def _rank_main(rank, world, init, q, mode):
    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from elffuss_engine_b200.ops import QuantOps
        from elffuss_engine_b200.tp import TPComm
        ops = QuantOps(rank)
        if mode == "timeout":
            comm = TPComm(ops, rank, world, max_bytes=4096, timeout_s=0.2)
            if rank == 0:                      # rank 1 never makes this call
                x = torch.ones(16, device="cuda")
                comm.all_reduce(x)
                torch.cuda.synchronize()
                st = comm.status()
                y = (torch.arange(4, device="cuda") * 2).tolist()      # the context still works
                q.put((rank, st, y))
            else:
                q.put((rank, 0, None))
            dist.barrier()
            comm.close()
            return
        comm = TPComm(ops, rank, world, max_bytes=1 << 16)
        if mode == "gather":
            import ctypes
            from elffuss_engine_b200 import formats
            from elffuss_engine_b200._lib import check, lib
            L, h = lib(), ops.ctx.bind()
            P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
            out = []
            for n, k, M, t in ((256, 512, 1, "Q8_0"), (512, 1024, 3, "Q4_K"), (384, 512, 16, "Q8_0")):
                raw = formats.synth(t, n, k, seed=20 + rank + n)    # this rank's rows of the whole matrix
                w = ops.load_weight(t, raw, n, k)
                x = torch.randn(M, k, device="cuda", generator=torch.Generator("cuda").manual_seed(5))
                y = torch.empty(M, n, device="cuda")
                ref = torch.empty(world * M * n, device="cuda")
                check(L.ef_gemv(h, w.h, P(x), M, P(y)), h)
                comm.all_gather(ref, y)
                got = []
                for rep in range(3):                 # repeated, and interleaved with the fused all-reduce
                    ya = torch.full((world * M * n,), float("nan"), device="cuda")
                    check(L.ef_gemv_allgather(h, comm.tp, w.h, P(x), M, P(ya)), h)
                    if rep == 1:
                        xr, nrm = torch.zeros(1, n, device="cuda"), torch.empty(1, n, device="cuda")
                        wn = torch.ones(n, device="cuda")
                        check(L.ef_gemv_allreduce_norm(h, comm.tp, w.h, P(x), 1, None, P(xr), P(wn),
                                                       ctypes.c_float(1e-5), P(nrm)), h)
                    got.append(ya)
                torch.cuda.synchronize()
                # numpy arrays travel through the queue by value (tensors would be shared
                # through file descriptors of a process that may already have exited)
                out.append((ref.cpu().numpy(), [g.cpu().numpy() for g in got]))
                w.free()
            q.put((rank, comm.status(), out))
            dist.barrier()
            comm.close()
            return
        if mode == "fused":
            import ctypes
            import numpy as np
            from elffuss_engine_b200 import formats
            from elffuss_engine_b200._lib import check, lib
            L, h = lib(), ops.ctx.bind()
            P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
            n, k, M = 256, 512, 3                          # this rank's k columns of a 256-row weight
            raw = formats.quantize_q8_0(np.random.default_rng(10 + rank).standard_normal((n, k)).astype(np.float32)
                                        * 0.05)
            w = ops.load_weight("Q8_0", raw, n, k)
            g = torch.Generator("cuda").manual_seed(7 + rank)
            x = torch.randn(M, k, device="cuda", generator=g)
            gen = torch.Generator("cuda").manual_seed(99)     # the same residual and norms on every rank
            resid0 = torch.randn(M, n, device="cuda", generator=gen)
            wp = torch.rand(n, device="cuda", generator=gen) + 0.5
            wn = torch.rand(n, device="cuda", generator=gen) + 0.5
            out = {}
            for fused in (True, False):
                for w_post in (wp, None):
                    xr = resid0.clone()
                    nrm = torch.empty(M, n, device="cuda")
                    if fused:
                        for _ in range(3):                     # repeated calls: parities and counters cycle
                            xr.copy_(resid0)
                            check(L.ef_gemv_allreduce_norm(h, comm.tp, w.h, P(x), M, P(w_post), P(xr), P(wn),
                                                           ctypes.c_float(1e-5), P(nrm)), h)
                    else:
                        o = torch.empty(M, n, device="cuda")
                        check(L.ef_gemv(h, w.h, P(x), M, P(o)), h)
                        comm.all_reduce(o)
                        check(L.ef_norm_add_norm(h, P(o), P(w_post), P(xr), P(wn), M, n, ctypes.c_float(1e-5),
                                                 P(nrm)), h)
                    torch.cuda.synchronize()
                    out[(fused, w_post is not None)] = (xr.cpu(), nrm.cpu())
            q.put((rank, comm.status(), out))
            dist.barrier()
            comm.close()
            return
        g = torch.Generator("cuda").manual_seed(100 + rank)
        xs = [torch.randn(n, device="cuda", generator=g) for n in (2048, 7, 4096)]
        inputs = [x.clone() for x in xs]
        for x in xs:
            comm.all_reduce(x)
        # any 4-byte word travels unchanged (-1 is all ones, 0x7fc00001 a NaN payload)
        pair = torch.tensor([rank * 10 + 1, -1 - rank, 0x7fc00001], dtype=torch.int32, device="cuda")
        gathered = torch.zeros(3 * world, dtype=torch.int32, device="cuda")
        comm.all_gather(gathered, pair)
        # the same calls replayed from a graph
        gx = torch.zeros(2048, device="cuda")
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s, capture_error_mode="thread_local"):
            comm.all_reduce(gx)
            comm.all_reduce(gx)
        torch.cuda.synchronize()
        replays = []
        for k in range(3):
            gx.fill_(float(rank + 1 + k))
            graph.replay()
            torch.cuda.synchronize()
            replays.append(gx[:4].tolist())
        del graph
        torch.cuda.synchronize()
        q.put((rank, comm.status(), [i.cpu() for i in inputs], [x.cpu() for x in xs], gathered.cpu().tolist(),
               replays))
        dist.barrier()
        comm.close()
    finally:
        dist.destroy_process_group()


def _run(mode):
    return run_ranks(_rank_main, 2, mode, timeout=180)


def test_allreduce_allgather_exact_and_graph_replay():
    got = _run("exact")
    for r in range(2):
        st, inputs, outs, gathered, replays = got[r]
        assert st == 0
        for j in range(3):
            want = got[0][1][j] + got[1][1][j]            # rank order: rank 0 + rank 1
            assert torch.equal(outs[j], want)
        assert gathered == [1, -1, 0x7fc00001, 11, -2, 0x7fc00001]
        for k in range(3):
            # two all-reduces of (1 + k) and (2 + k): (3 + 2k) * 2
            assert replays[k] == [float((3 + 2 * k) * 2)] * 4
    assert torch.equal(got[0][2][0], got[1][2][0])


def test_fused_gemv_allreduce_norm_equals_the_separate_calls():
    got = _run("fused")
    for r in range(2):
        st, out = got[r]
        assert st == 0
        for post in (True, False):
            xf, nf = out[(True, post)]
            xs, ns = out[(False, post)]
            assert torch.equal(xf, xs) and torch.equal(nf, ns)
            assert torch.equal(xf, got[0][1][(True, post)][0])      # the same bits on both ranks


def test_missing_rank_times_out_with_status():
    got = _run("timeout")
    st, y = got[0]
    assert st == -8                      # EF_ERR_TIMEOUT
    assert y == [0, 2, 4, 6]


def test_fused_gemv_allgather_equals_gemv_then_allgather():
    got = _run("gather")
    for r in range(2):
        st, out = got[r]
        assert st == 0
        for ref, reps in out:
            for g in reps:
                assert (g.view("u4") == ref.view("u4")).all()             # the same bits
        assert all((a[0].view("u4") == b[0].view("u4")).all() for a, b in zip(got[0][1], got[1][1]))
