"""Benchmark of the quantized GEMV hot path (BASELINE.json metric / config 1).

Workload (config 1, the K-quant GEMV sweep): Q4_K and Q6_K weights of shapes
14336x4096 and 4096x14336, activations M in {1, 4, 16} -- 12 GEMVs per round,
each on its OWN copy of its weight tensor; a step is ROUNDS = 8 rounds on 8
distinct copies (96 tensors, 3.9 GB: far more than the 126 MB L2, so every
GEMV reads HBM and no flush is needed). Synthetic seeded inputs with the
BASELINE.json distributions (no dataset exists).

  value  = algorithmic bytes of the step's 96 GEMVs (weights + x + y) / device
           time of the step: the step is captured once as a CUDA graph and
           replayed K times back to back; CUDA events around the K replays,
           inputs resident;
  e2e    = the same bytes through the public operator (QuantOps.gemv.matmul)
           with the step's x copied from pinned host memory and all its y
           copied back to pinned host memory inside every step;
  roofline: each call's GEMV launched back to back on its 8 weight copies,
           200 graph replays, against the measured HBM copy bandwidth
           (MEASURED_PEAKS.json).

N > 1 (torchrun, one rank per GPU): strong scaling -- every matrix of the
sweep is split by output rows over the ranks, each rank runs the GEMV on its
rows and an all-gather (the library's peer-memory collective, or NCCL with
--tp-comm nccl) assembles the whole y on every rank after every GEMV; value =
whole-matrix bytes / the max over ranks of the step time. The weak-scaling
figure (every rank streaming its own whole tensors) is reported beside it.

--impl reference: the reference's CPU arithmetic restated in C (oracle/, the
reference's own CPU path needs a JavaScript engine with WebAssembly, which is
absent here and on the GPU box) on all host cores, on a bounded row sample of
the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [(14336, 4096), (4096, 14336)]
TYPES = ["Q4_K", "Q6_K"]
MS = [1, 4, 16]
METRIC = "quant GEMV GB/s (% of HBM peak)"
WORKLOAD = "config1 K-quant GEMV sweep: {Q4_K,Q6_K} x {14336x4096, 4096x14336} x M{1,4,16}"


def calls():
    return [(t, n, k, m) for t in TYPES for (n, k) in SHAPES for m in MS]


def alg_bytes(t, n, k, m):
    from elffuss_engine_b200 import formats
    return formats.tensor_bytes(t, n, k) + 4 * m * k + 4 * m * n


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic():
    """DRAM read+write bytes of one step's 12 GEMV launches, from the committed ncu launch list."""
    path = os.path.join(ROOT, "profiles", "gemv_ksweep_launches.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_step:"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.samples, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def cpu_sample(threads: int, budget_s: float):
    """The oracle's f32 GEMV (the reference's CPU arithmetic, restated) on a row
    sample of every call of the workload; returns (GB/s, description)."""
    import numpy as np

    import oracle
    from elffuss_engine_b200 import formats
    rows_s = 512
    done_bytes, t_used = 0, 0.0
    sample_desc = f"{rows_s} rows of each of the 12 GEMVs (all k, all tokens), repeated for ~{budget_s:.0f}s"
    data = []
    for (t, n, k, m) in calls():
        raw = formats.synth(t, rows_s, k, seed=n + k)
        x = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
        data.append((t, k, m, raw, x))
    t_end = time.perf_counter() + budget_s
    while True:
        for (t, k, m, raw, x) in data:
            t0 = time.perf_counter()
            oracle.matmul_f32(t, raw, rows_s, k, x, tokens=m, threads=threads)
            t_used += time.perf_counter() - t0
            done_bytes += raw.size + 4 * m * k + 4 * m * rows_s
        if time.perf_counter() >= t_end:
            break
    return done_bytes / t_used / 1e9, sample_desc


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle
    oracle.build()
    threads = os.cpu_count() or 1
    vals = []
    for i in range(args.warmup + args.steps):
        v, desc = cpu_sample(threads, budget_s=2.0)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": sweep_config(args.gpus, ROUNDS * sum(alg_bytes(*c) for c in calls())),
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference CPU path (js/cpu.js + WASM) needs node, absent; its WebGPU path is unavailable "
                    "on this box; timed: the C restatement of its arithmetic"}
    print(json.dumps(line), flush=True)
    return 0


GEMM_SHAPES = [(512, 2048, 8192), (2048, 8192, 2048)]   # (tokens M, k, weight rows N)


def bench_gemm(ops, L, args, capture, timed_replays, rank):
    """Config 2: f16 activations x Q8_0 weights through ef_gemm, graph-replayed
    REPLAYS times; 8 distinct weight tensors per shape (more than L2 per replay)."""
    import torch

    from elffuss_engine_b200 import formats
    from elffuss_engine_b200._lib import check
    from elffuss_engine_b200.ops import _ptr
    peak, sustained = 1590.0, 1400.0
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            mp = json.load(f)
        peak, sustained = float(mp["bf16_tflops"]), float(mp["bf16_tflops_sustained"])
        src = "measured (dense bf16 burst; frac_sustained: against the sustained figure)"
    except Exception:
        src = "fallback"
    per_shape, tot_flop, tot_ms = [], 0.0, 0.0
    for si, (m, k, n) in enumerate(GEMM_SHAPES):
        raw = formats.synth("Q8_0", n, k, seed=500 + si + 10 * rank)
        ws = [ops.load_weight("Q8_0", raw, n, k) for _ in range(8)]
        del raw
        x = torch.randn(m, k, device="cuda", generator=torch.Generator("cuda").manual_seed(si)).half()
        y = torch.empty(m, n, device="cuda")

        def step():
            h = ops.ctx.bind()
            for w in ws:
                check(L.ef_gemm(h, w.h, _ptr(x), 1, m, _ptr(y), 0), h)
        step()
        g = capture(step)
        for _ in range(args.warmup):
            g.replay()
        ms = timed_replays(g, REPLAYS) / (REPLAYS * len(ws))
        del g
        flop = 2.0 * m * n * k
        tot_flop += flop
        tot_ms += ms
        per_shape.append({"M": m, "K": k, "N": n, "us": round(ms * 1e3, 2),
                          "TFLOPs": round(flop / (ms * 1e-3) / 1e12, 1),
                          "frac": round(flop / (ms * 1e-3) / 1e12 / peak, 4),
                          "frac_sustained": round(flop / (ms * 1e-3) / 1e12 / sustained, 4)})
        del ws, x, y
    torch.cuda.empty_cache()
    ach = tot_flop / (tot_ms * 1e-3) / 1e12
    return {"workload": "config2 Q8_0 prefill GEMM (tcgen05): M=512,K=2048,N=8192 and M=2048,K=8192,N=2048; "
                        "f16 activations, f32 out; 8 distinct weight tensors per shape",
            "per_shape": per_shape,
            "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(ach / peak, 4), "peak_sustained": sustained,
                         "frac_sustained": round(ach / sustained, 4), "peak_source": src,
                         "kernel": "ef_gemm_q8_0_kernel"}}


DECODE_PROMPT, DECODE_TOKENS = 512, 128
_COMM = {}


def tp_comm(ops, args, world, rank):
    """The decoders' collectives for world > 1: the library's peer-memory
    kernels (tp.TPComm, default) or NCCL (--tp-comm nccl)."""
    if world == 1 or args.tp_comm == "nccl":
        return None
    if "c" not in _COMM:
        from elffuss_engine_b200.tp import TPComm
        _COMM["c"] = TPComm(ops, rank, world, max_bytes=1 << 20)
    return _COMM["c"]


def bench_decode(ops, args, world, rank, barrier, max_over_ranks):
    """Config 3: the synthetic LFM3-shaped decoder (lfm3.py), tensor-parallel
    over the ranks when world > 1: a 512-id prompt (all ids at once through
    the GEMM path), then 128 greedy tokens, each one replay of the captured
    step."""
    import torch

    from elffuss_engine_b200.lfm3 import LFM3Config, LFM3Decoder, shard_weights, synth_weights
    cfg = LFM3Config()
    w = synth_weights(cfg, seed=0, device="cuda")
    if world > 1:
        w = shard_weights(cfg, w, rank, world)
    dec = LFM3Decoder(ops, cfg, w, rank, world, comm=tp_comm(ops, args, world, rank),
                      fused=world > 1 and args.tp_comm == "peer")
    del w
    torch.cuda.empty_cache()
    prompt = torch.randint(0, cfg.vocab, (DECODE_PROMPT,), generator=torch.Generator().manual_seed(0),
                           dtype=torch.int32).pin_memory()
    total = DECODE_PROMPT + DECODE_TOKENS
    # warm-up: eager step, the whole prompt (sizes the GEMM scratch), capture, a few steps
    dec.generate(prompt, 4, use_graph=True)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    tokens_h = torch.empty(DECODE_TOKENS + 1, dtype=torch.int32).pin_memory()
    dec.reset(out_base=DECODE_PROMPT)
    dec.capture()                                         # the step with this run's token offset
    barrier()
    ev[0].record()
    prompt_d = prompt.to(dec.tok.device, non_blocking=True)   # prompt ids host -> device
    dec.prefill(prompt_d)                                 # the whole prompt through the GEMM path
    ev[1].record()
    for _ in range(DECODE_TOKENS):
        dec.run_step()
    ev[2].record()
    tokens_h.copy_(dec.out_tokens[:DECODE_TOKENS + 1], non_blocking=True)   # tokens device -> host
    ev[3].record()
    barrier()
    prefill_ms = max_over_ranks(ev[0].elapsed_time(ev[1]))
    decode_ms = max_over_ranks(ev[1].elapsed_time(ev[2]))
    e2e_ms = max_over_ranks(ev[0].elapsed_time(ev[3]))
    toks = tokens_h.tolist()
    weight_bytes = cfg.weight_params() * 34 // 32
    dec.graph = None
    del dec
    torch.cuda.empty_cache()
    return {"workload": f"config3 synthetic LFM3-shaped decoder (Q8_0, hidden 2048, 16 layers: 10 short-conv + "
                        f"6 GQA at {list(cfg.attn_layers)}), {DECODE_PROMPT}-id prompt (one batched pass through the "
                        f"GEMM path) then {DECODE_TOKENS} greedy steps, each step one CUDA-graph replay",
            "parallelism": f"tp{world} ({args.tp_comm} collectives)" if world > 1 else "single GPU",
            "tok_s": round(DECODE_TOKENS / (decode_ms * 1e-3), 1),
            "ms_per_token": round(decode_ms / DECODE_TOKENS, 4),
            "weight_GBps_per_gpu": round(weight_bytes / world / (decode_ms / DECODE_TOKENS * 1e-3) / 1e9, 1),
            "prefill_ms": round(prefill_ms, 2),
            "e2e": {"tok_s": round(DECODE_TOKENS / (e2e_ms * 1e-3), 1), "ms": round(e2e_ms, 2),
                    "what": "prompt ids host->device, the prompt pass, greedy steps, tokens device->host",
                    "h2d_bytes": 4 * DECODE_PROMPT, "d2h_bytes": 4 * (DECODE_TOKENS + 1)},
            "first_tokens": toks[:8]}


LLAMA_CONTEXT, LLAMA_STEPS = 4096, 32


def bench_llama(ops, args, world, rank, barrier, max_over_ranks):
    """Config 4: the synthetic Llama-architecture 8B-shaped decoder (llama.py,
    Q4_K with Q6_K for attn_v, even-layer ffn_down and the head),
    tensor-parallel over the ranks when world > 1: a 4096-id context (its
    first 4095 ids through the GEMM path once), then greedy decode steps at
    batch 1 and at batch 16 (16 sequences sharing the first 4095 ids, each
    with its own last id), each step one CUDA-graph replay; batch 16 again
    with f16 KV caches (the reference's kvF16 option)."""
    import torch

    from elffuss_engine_b200.llama import LlamaConfig, LlamaDecoder, shard_weights, synth_weights
    cfg = LlamaConfig()
    w = synth_weights(cfg, seed=0, device="cuda")
    if world > 1:
        w = shard_weights(cfg, w, rank, world)
    ids = torch.randint(0, cfg.vocab, (LLAMA_CONTEXT + 15,), generator=torch.Generator().manual_seed(4),
                        dtype=torch.int32)
    prompt = ids[:LLAMA_CONTEXT]
    out = {"workload": f"config4 synthetic Llama-architecture 8B shape (32 layers, hidden 4096, 32/8 heads x 128, "
                       f"FFN 14336, vocab 128256; Q4_K, Q6_K for attn_v / even ffn_down / output), "
                       f"{LLAMA_CONTEXT}-id context, {LLAMA_STEPS} greedy steps per batch size",
           "parallelism": f"tp{world} ({args.tp_comm} collectives)" if world > 1 else "single GPU",
           "weight_bytes_per_step_per_gpu": cfg.step_weight_bytes() // world}
    import dataclasses
    for B, kv16 in ((1, False), (16, False), (16, True)):
        dec = LlamaDecoder(ops, dataclasses.replace(cfg, kv_f16=kv16), w, batch=B, rank=rank, world=world,
                           comm=tp_comm(ops, args, world, rank), fused=world > 1 and args.tp_comm == "peer")
        lasts = [int(prompt[-1])] + [int(t) for t in ids[LLAMA_CONTEXT:LLAMA_CONTEXT + B - 1]]
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        barrier()
        ev[0].record()
        dec.start(prompt, lasts)
        ev[1].record()
        barrier()
        prefill_ms = max_over_ranks(ev[0].elapsed_time(ev[1]))
        dec.step()                                           # eager: sizes scratch, configures kernels
        torch.cuda.synchronize()
        dec.rewind(LLAMA_CONTEXT, lasts)
        dec.capture()
        for _ in range(2):                                   # warm-up replays (positions advance)
            dec.run_step()
        barrier()
        ev[1].record()
        for _ in range(LLAMA_STEPS):
            dec.run_step()
        ev[2].record()
        barrier()
        ms = max_over_ranks(ev[1].elapsed_time(ev[2])) / LLAMA_STEPS
        toks = dec.out_tokens[:, :4].cpu().tolist()
        out[f"batch{B}" + ("_kv_f16" if kv16 else "")] = {"tok_s": round(B * 1e3 / ms, 1), "ms_per_step": round(ms, 4),
                            "weight_GBps_per_gpu": round(cfg.step_weight_bytes() / world / (ms * 1e-3) / 1e9, 1),
                            "prefill_4095_ms": round(prefill_ms, 1), "first_tokens": toks[0][:4],
                            "distinct_first_tokens": len({t[0] for t in toks})}
        dec.graph = None
        del dec
        torch.cuda.empty_cache()
    del w
    torch.cuda.empty_cache()
    return out


TRACE_SHAPES = [("Q4_K", 14336, 4096, 1), ("Q4_K", 4096, 14336, 1), ("Q6_K", 14336, 4096, 1),
                ("Q6_K", 4096, 14336, 1), ("Q8_0", 8192, 2048, 1), ("Q8_0", 2048, 2048, 1)]


def run_gemv_trace(args):
    """Launch phases of the GEMV kernel (needs `build.py --trace`): for each
    shape, ROUNDS weight copies launched back to back in a CUDA graph (as
    per_call), one replay traced. Per launch: the gap between the previous
    launch's last CTA exit and this launch's wait release, and per CTA (SM
    cycle counts, median over CTAs and launches 1..) the time before the wait
    returns, the activation staging, the weight stream and the epilogue.
    Prints one JSON line."""
    import ctypes

    import numpy as np
    import torch

    import elffuss_engine_b200._lib as _libmod
    _libmod.LIB_PATH = os.path.join(os.path.dirname(_libmod.LIB_PATH), "libelffuss_cuda_trace.so")
    from elffuss_engine_b200 import formats
    from elffuss_engine_b200._lib import check, lib
    from elffuss_engine_b200.ops import QuantOps, _ptr
    L = lib()
    L.ef_gemv_trace_set.argtypes = [ctypes.c_void_p, ctypes.c_uint]
    L.ef_gemv_trace_set.restype = ctypes.c_int
    ops = QuantOps(0)
    cap = 1 << 14
    buf = torch.zeros(cap * 12, dtype=torch.int64, device="cuda")
    ghz = torch.cuda.get_device_properties(0).clock_rate / 1e6 if hasattr(torch.cuda.get_device_properties(0),
                                                                           "clock_rate") else 1.965
    out = []
    for t, n, k, m in TRACE_SHAPES:
        raw = formats.synth(t, n, k, seed=5)
        ws = [ops.load_weight(t, raw, n, k) for _ in range(ROUNDS)]
        x = torch.randn(m, k, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
        y = torch.empty(m, n, device="cuda")

        def seq():
            h = ops.ctx.bind()
            for wc in ws:
                check(L.ef_gemv(h, wc.h, _ptr(x), m, _ptr(y)), h)
        cs = torch.cuda.Stream()
        cs.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cs):
            seq()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cs):
            seq()
        for _ in range(20):
            g.replay()
        buf.zero_()
        torch.cuda.synchronize()
        assert L.ef_gemv_trace_set(ctypes.c_void_p(buf.data_ptr()), cap) == 0
        g.replay()
        torch.cuda.synchronize()
        assert L.ef_gemv_trace_set(None, 0) == 0
        tr = buf.view(cap, 12).cpu().numpy()
        tr = tr[tr[:, 2] > 0]
        tr = tr[np.lexsort((tr[:, 2], tr[:, 0]))]
        launch = np.zeros(len(tr), dtype=int)
        for b in np.unique(tr[:, 0]):
            idx = np.where(tr[:, 0] == b)[0]
            launch[idx] = np.arange(len(idx))
        ctas = len(tr) // ROUNDS
        cyc = lambda a, b: float(np.median((tr[launch >= 1, 7 + b] - tr[launch >= 1, 7 + a]) / ghz / 1e3))
        ends = [tr[launch == i, 6].max() for i in range(ROUNDS)]
        waits = [tr[launch == i, 3].min() for i in range(ROUNDS)]
        period = (tr[launch == ROUNDS - 1, 2].min() - tr[launch == 1, 2].min()) / (ROUNDS - 2) / 1e3
        out.append({"shape": f"{t} {n}x{k} M={m}", "ctas": ctas, "period_us": round(period, 2),
                    "release_after_prev_exit_us": round(float(np.median(
                        [(waits[i + 1] - ends[i]) / 1e3 for i in range(ROUNDS - 1)])), 2),
                    "before_wait_us": round(cyc(0, 1), 2), "staging_us": round(cyc(1, 2), 2),
                    "stream_us": round(cyc(2, 3), 2), "epilogue_us": round(cyc(3, 4), 2)})
        del g
        for wc in ws:
            wc.free()
    print(json.dumps({"gemv_trace": out, "sm_ghz": ghz}), flush=True)
    return 0


def run_attn_probe(args):
    """Decode attention alone at config 4's batch-16 shape (16 sequences at
    position 4095, 32 query / 8 cache heads of 128, caches of LlamaConfig's
    capacity), f32 and f16 caches: 8 layers' calls (distinct caches) captured
    in a CUDA graph, 20 replays; per call time and K/V bytes read per second.
    Prints one JSON line."""
    import ctypes

    import torch

    from elffuss_engine_b200._lib import check, lib
    from elffuss_engine_b200.llama import LlamaConfig
    from elffuss_engine_b200.ops import QuantOps
    cfg = LlamaConfig()
    ops = QuantOps(0)
    L = lib()
    S, H, KV, D, maxp, layers = 16, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.max_pos, 8
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    out = {}
    for kv16 in (False, True):
        dt = torch.float16 if kv16 else torch.float32
        g = torch.Generator("cuda").manual_seed(1)
        kc = [torch.randn(S, maxp, KV, D, device="cuda", generator=g).to(dt) for _ in range(layers)]
        vc = [torch.randn(S, maxp, KV, D, device="cuda", generator=g).to(dt) for _ in range(layers)]
        q = torch.randn(S, H * D, device="cuda", generator=g)
        pos = torch.full((S,), LLAMA_CONTEXT - 1, dtype=torch.int32, device="cuda")
        o = torch.empty(S, H * D, device="cuda")
        fn = L.ef_attention_f16 if kv16 else L.ef_attention

        def seq():
            h = ops.ctx.bind()
            for i in range(layers):
                check(fn(h, P(q), P(kc[i]), P(vc[i]), None, P(pos), S, 1, maxp, 0, H, KV, D, P(o)), h)
        seq()
        torch.cuda.synchronize()
        cs = torch.cuda.Stream()
        cs.wait_stream(torch.cuda.current_stream())
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=cs):
            seq()
        for _ in range(3):
            gr.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(20):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / (20 * layers) * 1e3
        kv_bytes = 2 * S * LLAMA_CONTEXT * KV * D * (2 if kv16 else 4)
        out["f16" if kv16 else "f32"] = {"us_per_layer": round(us, 1), "kv_bytes": kv_bytes,
                                         "GBps": round(kv_bytes / us / 1e3, 1),
                                         "ms_per_step_32_layers": round(us * cfg.layers / 1e3, 3)}
        del gr, kc, vc
        torch.cuda.empty_cache()
    print(json.dumps({"attn_probe": out, "shape": f"S={S} pos={LLAMA_CONTEXT - 1} H={H} KVH={KV} D={D}"}),
          flush=True)
    return 0


def run_profile(args):
    """Profiling drivers for ncu (no timing): --ncu-gemm runs config 2's first
    GEMM shape (M=512, K=2048, N=8192) on 4 weight copies, eagerly, 3 times;
    --ncu-decode builds the config-3 LFM3 decoder and runs 8 eager decode
    steps, the last inside an NVTX range named "step"."""
    import torch

    import __graft_entry__
    __graft_entry__.package()
    from elffuss_engine_b200 import formats
    from elffuss_engine_b200._lib import check, lib
    from elffuss_engine_b200.ops import QuantOps, _ptr
    ops, L = QuantOps(0), lib()
    if args.ncu_gemm:
        m, k, n = GEMM_SHAPES[0]
        raw = formats.synth("Q8_0", n, k, seed=500)
        ws = [ops.load_weight("Q8_0", raw, n, k) for _ in range(4)]
        x = torch.randn(m, k, device="cuda", generator=torch.Generator("cuda").manual_seed(0)).half()
        y = torch.empty(m, n, device="cuda")
        for _ in range(3):
            h = ops.ctx.bind()
            for w in ws:
                check(L.ef_gemm(h, w.h, _ptr(x), 1, m, _ptr(y), 0), h)
        torch.cuda.synchronize()
        print(json.dumps({"ncu_gemm": True, "launches": 12}), flush=True)
        return 0
    from elffuss_engine_b200.lfm3 import LFM3Config, LFM3Decoder, synth_weights
    cfg = LFM3Config()
    dec = LFM3Decoder(ops, cfg, synth_weights(cfg, seed=0, device="cuda"))
    dec.reset(out_base=0)
    for i in range(8):
        dec.tok.fill_(i)
        if i == 7:
            torch.cuda.nvtx.range_push("step")
        dec.step()
        if i == 7:
            torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(json.dumps({"ncu_decode": True}), flush=True)
    return 0


ROUNDS = 8          # weight copies per call: a step streams every call's matrix ROUNDS times
REPLAYS = 200       # graph replays behind each per-call duration


def sweep_config(world: int, step_bytes: int) -> dict:
    """The `config` object of both arms' JSON lines (same keys)."""
    return {"workload": WORKLOAD, "rounds_per_step": ROUNDS, "bytes_per_step": step_bytes,
            "l2": f"inputs larger than L2: {ROUNDS} distinct weight tensors per call, "
                  f"{ROUNDS * 12} per step ({ROUNDS * 486} MB at N = 1)",
            "parallelism": "single GPU" if world == 1 else
            f"row-sharded x{world}: every matrix split by output rows over the ranks, y assembled on every "
            f"rank by an all-gather of each GEMV's output (fused into the GEMV with the peer collectives)"}


def shard_rows(raw, t: str, n: int, k: int, rank: int, world: int):
    """Rows [rank * n / world, (rank + 1) * n / world) of a GGUF tensor's bytes."""
    from elffuss_engine_b200 import formats
    per_row = formats.tensor_bytes(t, 1, k)
    r0, r1 = rank * n // world, (rank + 1) * n // world
    return raw.reshape(-1)[r0 * per_row:r1 * per_row], r1 - r0


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    import __graft_entry__
    __graft_entry__.package()
    from elffuss_engine_b200 import formats
    from elffuss_engine_b200._lib import check, lib
    from elffuss_engine_b200.ops import QuantOps, _ptr

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device(f"cuda:{local}"))
    ops = QuantOps(local)
    L = lib()
    comm = tp_comm(ops, args, world, rank) if world > 1 else None

    # weights: ROUNDS tensors per call (this rank's row shard of each at N > 1),
    # each drawn by the seeded host generator with the BASELINE distributions;
    # the same x per call in every round.
    work = []
    for i, (t, n, k, m) in enumerate(calls()):
        raw = formats.synth(t, n, k, seed=i)
        part, rows = shard_rows(raw, t, n, k, rank, world) if world > 1 else (raw, n)
        ws = [ops.load_weight(t, part, rows, k) for _ in range(ROUNDS)]
        x = torch.randn(m, k, device="cuda", generator=torch.Generator("cuda").manual_seed(i))
        y = torch.empty(m, rows, device="cuda")
        yall = torch.empty(world * m * rows, device="cuda") if world > 1 else None
        work.append(dict(t=t, n=n, k=k, m=m, rows=rows, ws=ws, x=x, y=y, yall=yall,
                         bytes=alg_bytes(t, n, k, m), shard_bytes=alg_bytes(t, rows, k, m)))
    del raw, part
    step_bytes = ROUNDS * sum(wk["bytes"] for wk in work)        # whole matrices (all ranks together)

    def gather(wk):
        if world > 1:
            if comm is not None:
                comm.all_gather(wk["yall"], wk["y"])
            else:
                dist.all_gather_into_tensor(wk["yall"], wk["y"].view(-1))

    def step_device():
        h = ops.ctx.bind()
        for r in range(ROUNDS):
            for wk in work:
                if world > 1 and comm is not None:   # the GEMV and its all-gather fused
                    check(L.ef_gemv_allgather(h, comm.tp, wk["ws"][r].h, _ptr(wk["x"]), wk["m"], _ptr(wk["yall"])), h)
                else:
                    check(L.ef_gemv(h, wk["ws"][r].h, _ptr(wk["x"]), wk["m"], _ptr(wk["y"])), h)
                    gather(wk)

    # end-to-end buffers: the step's inputs in one pinned host buffer (one
    # host->device copy per step), all its results gathered for one readback
    x_elems = sum(wk["m"] * wk["k"] for wk in work)
    y_elems = ROUNDS * sum(wk["m"] * wk["rows"] * world for wk in work)
    xh_all = torch.cat([wk["x"].view(-1).cpu() for wk in work]).pin_memory()
    x_all = torch.empty(x_elems, device="cuda")
    y_all = torch.empty(y_elems, device="cuda")
    yh_all = torch.empty(y_elems, dtype=torch.float32).pin_memory()
    x_views, off = [], 0
    for wk in work:
        x_views.append(x_all[off:off + wk["m"] * wk["k"]].view(wk["m"], wk["k"]))
        off += wk["m"] * wk["k"]

    copy_stream = torch.cuda.Stream()
    round_elems = y_elems // ROUNDS

    def step_e2e():
        x_all.copy_(xh_all, non_blocking=True)                  # the step's inputs, host -> device
        for r in range(ROUNDS):
            outs = []
            for wk, xv in zip(work, x_views):
                o = ops.gemv.matmul(wk["t"], wk["ws"][r], xv, wk["rows"], wk["k"], wk["m"])   # public operator
                if world > 1:
                    wk["y"].copy_(o)
                    gather(wk)
                    o = wk["yall"]
                outs.append(o.view(-1))
            seg = y_all[r * round_elems:(r + 1) * round_elems]
            torch.cat(outs, out=seg)
            # this round's results, device -> host, on a copy stream while the next round computes
            done = torch.cuda.Event()
            done.record()
            copy_stream.wait_event(done)
            with torch.cuda.stream(copy_stream):
                yh_all[r * round_elems:(r + 1) * round_elems].copy_(seg, non_blocking=True)
        torch.cuda.current_stream().wait_stream(copy_stream)   # the step ends with its results on the host

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        tv = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(tv, op=dist.ReduceOp.MAX)
        return float(tv.item())

    def capture(fn, *a):
        g = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream()
        cs.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cs):
            fn(*a)          # warm this stream (first-use attribute setup, scratch sizing)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=cs, capture_error_mode="thread_local"):
            fn(*a)
        torch.cuda.synchronize()
        return g

    def timed_replays(g, steps):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        ev0.record()
        for _ in range(steps):
            g.replay()
        ev1.record()
        barrier()
        return max_over_ranks(ev0.elapsed_time(ev1))

    # eager warm-up: kernel attributes and scratch sized before any capture
    for _ in range(args.warmup):
        step_device()
        if not args.ncu_step:
            step_e2e()
    barrier()
    n0 = L.ef_ctx_launch_count(ops.ctx.h)
    step_device()                     # one more eager step: count its kernel launches
    launches_per_step = L.ef_ctx_launch_count(ops.ctx.h) - n0
    barrier()
    if args.ncu_step:                 # profiling mode: warm-up + one counted eager step only
        if rank == 0:
            print(json.dumps({"ncu_step": True, "launches_per_step": launches_per_step,
                              "warmup_launches": launches_per_step * args.warmup}), flush=True)
        return 0

    with Clocks(local) as clk:
        # ---- device-resident timing: one captured step, replayed K times ----
        g_dev = capture(step_device)
        for _ in range(args.warmup):
            g_dev.replay()
        t_ms = timed_replays(g_dev, args.steps)
        ms_step = t_ms / args.steps
        value = step_bytes / (ms_step * 1e-3) / 1e9
        del g_dev

        # ---- per-kernel durations: each call's GEMV launched back to back on
        # its ROUNDS weight copies (more than L2 between reuses), CUDA events
        # around REPLAYS replays of that captured sequence ----
        kern_ms = []
        for wk in work:
            def seq(wk=wk):
                h = ops.ctx.bind()
                for wc in wk["ws"]:
                    check(L.ef_gemv(h, wc.h, _ptr(wk["x"]), wk["m"], _ptr(wk["y"])), h)
            g_k = capture(seq)
            g_k.replay()
            kern_ms.append(timed_replays(g_k, REPLAYS) / (REPLAYS * ROUNDS))
            del g_k

        # ---- config 0: Q8_0 GEMV 8192 x 2048, 1 token (the same back-to-back method) ----
        raw0 = formats.synth("Q8_0", 8192, 2048, seed=77)
        ws0 = [ops.load_weight("Q8_0", raw0, 8192, 2048) for _ in range(ROUNDS)]
        del raw0
        x0 = torch.randn(1, 2048, device="cuda", generator=torch.Generator("cuda").manual_seed(77))
        y0 = torch.empty(1, 8192, device="cuda")

        def seq0():
            h = ops.ctx.bind()
            for wc in ws0:
                check(L.ef_gemv(h, wc.h, _ptr(x0), 1, _ptr(y0)), h)
        g0 = capture(seq0)
        g0.replay()
        us0 = timed_replays(g0, REPLAYS) * 1e3 / (REPLAYS * ROUNDS)
        b0 = formats.tensor_bytes("Q8_0", 8192, 2048) + 4 * 2048 + 4 * 8192
        del g0
        for wc in ws0:
            wc.free()

        # ---- end to end through the public operator, pinned host buffers ----
        g_e2e = capture(step_e2e)
        for _ in range(args.warmup):
            g_e2e.replay()
        e2e_ms = timed_replays(g_e2e, args.steps) / args.steps
        e2e_val = step_bytes / (e2e_ms * 1e-3) / 1e9
        h2d = 4 * x_elems
        d2h = 4 * y_elems
        del g_e2e

    # ---- N > 1: the same sweep with every rank streaming its own whole tensors
    # (weak scaling, no collective), for comparison with the sharded value ----
    weak = None
    if world > 1:
        full = []
        for i, (t, n, k, m) in enumerate(calls()):
            raw = formats.synth(t, n, k, seed=1000 * rank + i)
            full.append((ops.load_weight(t, raw, n, k), torch.empty(m, n, device="cuda"), m, alg_bytes(t, n, k, m)))
        del raw

        def step_weak():
            h = ops.ctx.bind()
            for (w, y, m, b), wk in zip(full, work):
                check(L.ef_gemv(h, w.h, _ptr(wk["x"]), m, _ptr(y)), h)
        g_w = capture(step_weak)
        for _ in range(3):
            g_w.replay()
        wms = timed_replays(g_w, 10 * args.steps) / (10 * args.steps)
        weak = {"value": round(world * sum(b for *_, b in full) / (wms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(wms, 4), "scaling": "weak",
                "what": "every rank streams its own whole 12 tensors of the sweep, no collective; whole-job GB/s"}
        del g_w
        for w, *_ in full:
            w.free()

    # ---- config 2: Q8_0 prefill GEMM on tcgen05 (tensor roofline) ----
    gemm = None
    if not args.no_gemm:
        with Clocks(local) as gclk:
            gemm = bench_gemm(ops, L, args, capture, timed_replays, rank)
        gemm["clocks"] = gclk.summary()
    for wk in work:
        for w in wk["ws"]:
            w.free()
    torch.cuda.empty_cache()

    # ---- config 3: LFM3-shaped decode, tensor-parallel over the ranks ----
    decode = None if args.no_decode else bench_decode(ops, args, world, rank, barrier, max_over_ranks)
    decode8b = None if args.no_decode else bench_llama(ops, args, world, rank, barrier, max_over_ranks)

    # ---- roofline of the dominant kernel (the GEMV, on this rank's rows) ----
    peak, peak_kind = peaks()
    shard_step = sum(wk["shard_bytes"] for wk in work)
    kern_total_ms = sum(kern_ms)
    achieved = shard_step / (kern_total_ms * 1e-3) / 1e9
    per_call = [{"type": wk["t"], "rows": wk["rows"], "k": wk["k"], "M": wk["m"], "us": round(kern_ms[j] * 1e3, 2),
                 "GBps": round(wk["shard_bytes"] / (kern_ms[j] * 1e-3) / 1e9, 1)} for j, wk in enumerate(work)]

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        oracle.build()
        cores = os.cpu_count() or 1
        v, desc = cpu_sample(cores, budget_s=args.cpu_seconds)
        capped = max(1, min(8, cores // 2))
        vc, _ = cpu_sample(capped, budget_s=args.cpu_seconds / 2)
        cpu = {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": desc,
               "reference_thread_cap": {"threads": capped, "value": round(vc, 3),
                                        "rule": "min(8, cores / 2), the reference CPU pool's own cap "
                                                "(js/cpu.js:107-113)"}}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak" if world == 1 else "strong", "vs_baseline": None,
            "dtype": "s8 x u8 -> s32 (Q4_K/Q6_K weights, x as two int8 planes per 256-block), f32 scales",
            "data": "synthetic",
            "config": sweep_config(world, step_bytes),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "traffic": profile_traffic() if world == 1 else None, "algorithmic_bytes": shard_step,
                         "per": f"the 12 calls of a round on this rank's rows: sum of their algorithmic bytes / "
                                f"sum of their average launch durations (each call launched back to back on its "
                                f"{ROUNDS} weight copies, {REPLAYS} graph replays; for M > 2 the duration "
                                f"includes the call's activation-prep kernel)",
                         "kernel": "ef_gemv_kernel"},
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps * launches_per_step,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "weak_scaling": weak,
            "gemm": gemm,
            "config0": {"workload": f"config0 Q8_0 GEMV 8192x2048, 1 token ({ROUNDS} weight copies back to back, "
                                    f"{REPLAYS} graph replays)",
                        "us": round(us0, 2), "GBps": round(b0 / (us0 * 1e-6) / 1e9, 1),
                        "frac": round(b0 / (us0 * 1e-6) / 1e9 / peak, 4), "algorithmic_bytes": b0},
            "decode": decode,
            "decode_8b": decode8b,
            "per_call": per_call,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        if "c" in _COMM:
            torch.cuda.synchronize()
            _COMM.pop("c").close()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-gemm", action="store_true", help="skip the config-2 GEMM measurement")
    ap.add_argument("--no-decode", action="store_true", help="skip the config-3/4 decode measurements")
    ap.add_argument("--tp-comm", default="peer", choices=["peer", "peer-separate", "nccl"],
                    help="tensor-parallel decode collectives: the library's peer-memory kernels with the "
                         "row-parallel GEMV and its all-reduce fused (peer) or as separate kernels, or NCCL")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ncu-step", action="store_true",
                    help="profiling mode for ncu: eager warm-up steps plus one eager step, no timing")
    ap.add_argument("--ncu-gemm", action="store_true", help="profiling mode for ncu: config-2 GEMM calls only")
    ap.add_argument("--attn-probe", action="store_true",
                    help="decode attention alone at config 4's batch-16 shape, f32 and f16 caches")
    ap.add_argument("--gemv-trace", action="store_true",
                    help="launch phases of the GEMV kernel from the trace library (build.py --trace)")
    ap.add_argument("--ncu-decode", action="store_true",
                    help="profiling mode for ncu: config-3 decode steps, the last in an NVTX range 'step'")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    import __graft_entry__
    __graft_entry__.package()
    if args.impl == "reference":
        return run_reference(args)
    if args.ncu_gemm or args.ncu_decode:
        return run_profile(args)
    if args.gemv_trace:
        return run_gemv_trace(args)
    if args.attn_probe:
        return run_attn_probe(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
