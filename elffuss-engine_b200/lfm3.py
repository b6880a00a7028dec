"""Synthetic LFM3-shaped decoder driven through the quantized GEMV path.

The reference runs LFM3 (LiquidAI's hybrid of gated short convolutions and
grouped-query attention) in js/model.js: per layer an RMSNorm, either the
short-conv block (convBlock, js/model.js:758-794) or the attention block
(attnBlock, :853-983, with per-head QK-norm, NEOX RoPE, a sigmoid gate per
head and sliding-window layers), each followed by a post-norm, the residual,
the FFN norm, a SwiGLU FFN, its post-norm and the residual (feedForward,
:635-664); the head is the tied embedding on the final norm of the last token
(:1158-1171) and sampling is greedy (js/sample.js:95-99).

This module builds that network from seeded synthetic weights (N(0, 0.02),
quantized to Q8_0 with d = max|x|/127 and round-to-nearest-even; norm weights
1; the depthwise conv weights kept in f32 as GGUF keeps them) and runs one
token per step entirely on the device: every matrix product is this library's
GEMV (q/k/v/gate as one sections call, gate/up as one SwiGLU call, the LM head
over the 65536-row tied embedding), the rest are the library's decoder-step
kernels. Position and token live in device memory, so a step is captured once
as a CUDA graph and replayed per token.

Tensor parallel (one process per GPU, Megatron-style; the reference runs on
one device): shard_weights gives rank r of g its slices -- q/k/v/gate by
heads, shortconv.in_proj by channel (the B, C and x rows of the same
channels, so the depthwise conv stays local), ffn_gate/up by inner rows, the
LM head by vocabulary rows (column-parallel, no exchange); attn_output,
shortconv.out_proj and ffn_down by input columns (row-parallel), each
followed by an all-reduce of the hidden vector (the library's peer-memory
collectives of tp.TPComm, or NCCL through torch.distributed; either is
captured in the step's graph). The head ends with a local
argmax per rank and an all-gather of the (value, index) pairs, so the token is
the one a single argmax over the whole vocabulary picks.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import formats
from ._lib import EfError, check, lib

Q8_0 = formats.type_id("Q8_0")


@dataclass
class LFM3Config:
    hidden: int = 2048
    layers: int = 16
    attn_layers: tuple = (2, 5, 8, 10, 12, 14)   # the attention layers; the others are short-conv
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 64
    ffn: int = 8192
    vocab: int = 65536
    conv_k: int = 3
    rope_theta: float = 1e6
    window: int = 4096              # sliding window of every other attention layer (the first, third, ...)
    eps: float = 1e-5
    max_pos: int = 4096 + 1024      # KV-cache capacity
    kv_f16: bool = False            # f16 KV caches (the reference's kvF16 option), f32 by default

    def windows(self) -> dict:
        """window per attention layer (0 = global): alternating, starting with a sliding one."""
        return {l: (self.window if j % 2 == 0 else 0) for j, l in enumerate(self.attn_layers)}

    def weight_params(self) -> int:
        E, H, KV, D, F = self.hidden, self.heads, self.kv_heads, self.head_dim, self.ffn
        conv = 3 * E * E + E * E
        attn = H * D * E + 2 * KV * D * E + H * E + E * H * D
        n_att = len(self.attn_layers)
        return (self.layers - n_att) * conv + n_att * attn + self.layers * 3 * F * E + self.vocab * E


SMALL = dict(hidden=256, layers=4, attn_layers=(1, 3), heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1024,
             window=8, max_pos=96)


def quantize_q8_0_torch(w: torch.Tensor) -> torch.Tensor:
    """f32 [rows][k] -> Q8_0 bytes (uint8, same device): d = max|x|/127 stored
    as f16, q = round-half-even(x / d) in f32 -- the arithmetic of
    formats.quantize_q8_0."""
    b = w.reshape(-1, 32).float()
    amax = b.abs().amax(dim=1)
    d = amax / 127.0
    inv = torch.where(d > 0, 1.0 / torch.where(d > 0, d, torch.ones_like(d)), torch.zeros_like(d))
    q = torch.clamp(torch.round(b * inv[:, None]), -127, 127).to(torch.int8)
    out = torch.empty(b.shape[0], 34, dtype=torch.uint8, device=w.device)
    out[:, 0:2] = d.to(torch.float16).view(torch.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(torch.uint8)
    return out.reshape(-1)


def synth_weights(cfg: LFM3Config, seed: int = 0, device: str = "cpu") -> dict:
    """Named tensors of the network: Q8_0 bytes (uint8, 1-D) for the matrices,
    f32 for the conv kernels and the norms. Tensor i draws N(0, 0.02) from a
    generator seeded with seed * 1000 + i on `device`."""
    E, H, KV, D, F, V = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab
    out, idx = {}, [0]

    def normal(*shape):
        g = torch.Generator(device=device)
        g.manual_seed(seed * 1000 + idx[0])
        idx[0] += 1
        return torch.empty(*shape, device=device).normal_(0.0, 0.02, generator=g)

    def mat(name, rows, k):
        out[name] = (quantize_q8_0_torch(normal(rows, k)), rows, k)

    ones = lambda n: torch.ones(n, device=device)
    mat("token_embd", V, E)
    out["output_norm"] = ones(E)
    for l in range(cfg.layers):
        p = f"blk.{l}."
        out[p + "attn_norm"] = ones(E)
        out[p + "post_attention_norm"] = ones(E)
        out[p + "ffn_norm"] = ones(E)
        out[p + "post_ffw_norm"] = ones(E)
        if l in cfg.attn_layers:
            mat(p + "attn_q", H * D, E)
            mat(p + "attn_k", KV * D, E)
            mat(p + "attn_v", KV * D, E)
            mat(p + "attn_gate", H, E)
            mat(p + "attn_output", E, H * D)
            out[p + "attn_q_norm"] = ones(D)
            out[p + "attn_k_norm"] = ones(D)
        else:
            mat(p + "shortconv.in_proj", 3 * E, E)
            out[p + "shortconv.conv"] = normal(E, cfg.conv_k)
            mat(p + "shortconv.out_proj", E, E)
        mat(p + "ffn_gate", F, E)
        mat(p + "ffn_up", F, E)
        mat(p + "ffn_down", E, F)
    return out


def _q8_rows(raw: torch.Tensor, rows: int, k: int, ranges) -> torch.Tensor:
    """Q8_0 bytes of the rows [a, b) of each range, concatenated in order."""
    m = raw.reshape(rows, (k // 32) * 34)
    return torch.cat([m[a:b] for a, b in ranges]).reshape(-1).contiguous()


def _q8_cols(raw: torch.Tensor, rows: int, k: int, c0: int, c1: int) -> torch.Tensor:
    """Q8_0 bytes of the columns [c0, c1) (multiples of 32) of every row."""
    m = raw.reshape(rows, k // 32, 34)
    return m[:, c0 // 32:c1 // 32].reshape(-1).contiguous()


def shard_weights(cfg: LFM3Config, weights: dict, rank: int, world: int) -> dict:
    """Rank `rank` of `world`: the slices of synth_weights' tensors this rank
    holds (see the module docstring). token_embd stays whole (the embedding
    gather reads one row of it); "output" is this rank's vocabulary rows of it."""
    E, H, KV, D, F, V = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab
    g, r = world, rank
    for what, n in (("heads", H), ("kv_heads", KV), ("hidden", E), ("ffn", F), ("vocab", V)):
        if n % g:
            raise ValueError(f"tensor parallel over {g} ranks: {what}={n} does not split")
    Hl, KVl, Ec, Fl, Vl = H // g, KV // g, E // g, F // g, V // g
    for what, n in (("heads*head_dim", Hl * D), ("hidden", Ec), ("ffn", Fl)):
        if n % 32:
            raise ValueError(f"tensor parallel over {g} ranks: the {what} slice {n} is not a multiple of 32")
    out = {}
    for name, val in weights.items():
        short = name.split(".", 2)[-1] if name.startswith("blk.") else name
        if not isinstance(val, tuple):
            if short == "shortconv.conv":
                out[name] = val[r * Ec:(r + 1) * Ec].contiguous()
            else:
                out[name] = val
            continue
        raw, rows, k = val
        if short == "token_embd":
            out[name] = val
            out["output"] = (_q8_rows(raw, rows, k, [(r * Vl, (r + 1) * Vl)]), Vl, k)
        elif short == "attn_q":
            out[name] = (_q8_rows(raw, rows, k, [(r * Hl * D, (r + 1) * Hl * D)]), Hl * D, k)
        elif short in ("attn_k", "attn_v"):
            out[name] = (_q8_rows(raw, rows, k, [(r * KVl * D, (r + 1) * KVl * D)]), KVl * D, k)
        elif short == "attn_gate":
            out[name] = (_q8_rows(raw, rows, k, [(r * Hl, (r + 1) * Hl)]), Hl, k)
        elif short == "attn_output":
            out[name] = (_q8_cols(raw, rows, k, r * Hl * D, (r + 1) * Hl * D), rows, Hl * D)
        elif short == "shortconv.in_proj":
            rr = [(j * E + r * Ec, j * E + (r + 1) * Ec) for j in range(3)]
            out[name] = (_q8_rows(raw, rows, k, rr), 3 * Ec, k)
        elif short == "shortconv.out_proj":
            out[name] = (_q8_cols(raw, rows, k, r * Ec, (r + 1) * Ec), rows, Ec)
        elif short in ("ffn_gate", "ffn_up"):
            out[name] = (_q8_rows(raw, rows, k, [(r * Fl, (r + 1) * Fl)]), Fl, k)
        elif short == "ffn_down":
            out[name] = (_q8_cols(raw, rows, k, r * Fl, (r + 1) * Fl), rows, Fl)
        else:
            raise ValueError(f"no shard rule for {name}")
    return out


def _p(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


class LFM3Decoder:
    """The network, a step per token (see the module docstring). With
    world > 1, `weights` are this rank's shard_weights and the collectives go
    through torch.distributed's default (NCCL) process group."""

    def __init__(self, ops, cfg: LFM3Config, weights: dict, rank: int = 0, world: int = 1, pdl: bool = True,
                 comm=None, fused: bool = True):
        self.ops, self.cfg, self.L = ops, cfg, lib()
        self.rank, self.world, self.pdl, self.comm, self.fused = rank, world, pdl, comm, fused
        E, D = cfg.hidden, cfg.head_dim
        H, KV, F = cfg.heads // world, cfg.kv_heads // world, cfg.ffn // world
        self.Hl, self.KVl, self.Ec, self.Fl, self.Vl = H, KV, E // world, F, cfg.vocab // world
        dev = torch.device("cuda", ops.ctx.device)
        self.w, self.f32 = {}, {}
        for name, val in weights.items():
            if isinstance(val, tuple):
                raw, rows, k = val
                self.w[name] = ops.load_weight("Q8_0", raw.to(dev), rows, k, label=name)
            else:
                self.f32[name] = val.to(dev).float().contiguous()
        if world == 1:
            self.w["output"] = self.w["token_embd"]
        z = lambda *s: torch.zeros(*s, device=dev)
        self.x, self.nrm = z(E), z(E)
        self.bcx, self.conv_y = z(3 * self.Ec), z(self.Ec)
        self.o, self.sw, self.d = z(E), z(F), z(E)
        self.q, self.k, self.v, self.g, self.att = z(H * D), z(KV * D), z(KV * D), z(H), z(H * D)
        self.logits = z(self.Vl)
        self.pair = torch.zeros(2, dtype=torch.int32, device=dev)
        self.pairs = torch.zeros(2 * world, dtype=torch.int32, device=dev)
        self.state = {l: z(cfg.conv_k - 1, self.Ec) for l in range(cfg.layers) if l not in cfg.attn_layers}
        kvt = torch.float16 if cfg.kv_f16 else torch.float32
        self.kc = {l: torch.zeros(cfg.max_pos, KV, D, dtype=kvt, device=dev) for l in cfg.attn_layers}
        self.vc = {l: torch.zeros(cfg.max_pos, KV, D, dtype=kvt, device=dev) for l in cfg.attn_layers}
        sfx = "_f16" if cfg.kv_f16 else ""
        self._qk_rope = getattr(self.L, "ef_qk_norm_rope_cache" + sfx)
        self._attn_dec = getattr(self.L, "ef_attn_decode" + sfx)
        self._rope = getattr(self.L, "ef_rope_cache" + sfx)
        self._attn = getattr(self.L, "ef_attention" + sfx)
        self.tok = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.out_tokens = torch.full((cfg.max_pos,), -1, dtype=torch.int32, device=dev)
        self.out_base = 0
        self.windows = cfg.windows()
        self.graph = None

    def reset(self, out_base: int):
        for t in list(self.state.values()) + list(self.kc.values()) + list(self.vc.values()):
            t.zero_()
        self.pos.zero_()
        self.out_tokens.fill_(-1)
        self.out_base = out_base
        self.graph = None

    # -- one decode step (token self.tok at position self.pos) -----------------
    def _reduce(self, t: torch.Tensor):
        """Sum of the ranks' partial row-parallel outputs (in place): through
        the peer-memory collectives (tp.TPComm) when given, else NCCL."""
        if self.world > 1:
            if self.comm is not None:
                self.comm.all_reduce(t)
            else:
                import torch.distributed as dist
                dist.all_reduce(t)

    def _rowpar(self, h, w, xin, out, w_post, w_next):
        """out = w xin (this rank's columns), summed over the ranks; then x +=
        rmsnorm(out) * w_post and nrm = rmsnorm(x) * w_next. With the
        peer-memory collectives, one fused call (ef_gemv_allreduce_norm)."""
        L, eps = self.L, ctypes.c_float(self.cfg.eps)
        if self.world > 1 and self.comm is not None and self.fused:
            check(L.ef_gemv_allreduce_norm(h, self.comm.tp, w.h, _p(xin), 1, _p(w_post), _p(self.x), _p(w_next),
                                           eps, _p(self.nrm)), h)
            return
        check(L.ef_gemv(h, w.h, _p(xin), 1, _p(out)), h)
        self._reduce(out)
        check(L.ef_norm_add_norm(h, _p(out), _p(w_post), _p(self.x), _p(w_next), 1, self.cfg.hidden, eps,
                                 _p(self.nrm)), h)

    def step(self):
        """Queue one step; with pdl, its kernels are launched as a programmatic-
        dependent-launch chain (each scheduled while the previous one ends)."""
        L, h = self.L, self.ops.ctx.bind()
        check(L.ef_ctx_set_pdl(h, 1 if self.pdl else 0), h)
        try:
            self._step()
        finally:
            L.ef_ctx_set_pdl(h, 1)   # the context default

    def _step(self):
        L, cfg, h = self.L, self.cfg, self.ops.ctx.bind()
        E, D = cfg.hidden, cfg.head_dim
        H, KV = self.Hl, self.KVl
        W, f = self.w, self.f32
        eps = ctypes.c_float(cfg.eps)
        check(L.ef_gather_rmsnorm(h, W["token_embd"].h, _p(self.tok), 1, _p(f["blk.0.attn_norm"]), eps, _p(self.x),
                                  _p(self.nrm)), h)
        for l in range(cfg.layers):
            p = f"blk.{l}."
            if l in cfg.attn_layers:
                ws = (ctypes.c_void_p * 4)(W[p + "attn_q"].h.value, W[p + "attn_k"].h.value, W[p + "attn_v"].h.value,
                                           W[p + "attn_gate"].h.value)
                ys = (ctypes.c_void_p * 4)(self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), self.g.data_ptr())
                check(L.ef_gemv_sections(h, ctypes.cast(ws, ctypes.POINTER(ctypes.c_void_p)), 4, _p(self.nrm), 1,
                                         ctypes.cast(ys, ctypes.POINTER(ctypes.c_void_p))), h)
                check(self._qk_rope(h, _p(self.q), _p(self.k), _p(self.v), _p(f[p + "attn_q_norm"]),
                                              _p(f[p + "attn_k_norm"]), _p(self.pos), cfg.max_pos, H, KV, D,
                                              ctypes.c_float(cfg.rope_theta), eps, _p(self.kc[l]), _p(self.vc[l])), h)
                check(self._attn_dec(h, _p(self.q), _p(self.kc[l]), _p(self.vc[l]), _p(self.g), _p(self.pos),
                                       cfg.max_pos, self.windows[l], H, KV, D, _p(self.att)), h)
                out_w, out_x = W[p + "attn_output"], self.att
            else:
                check(L.ef_gemv(h, W[p + "shortconv.in_proj"].h, _p(self.nrm), 1, _p(self.bcx)), h)
                check(L.ef_shortconv(h, _p(self.bcx), _p(f[p + "shortconv.conv"]), _p(self.state[l]), 1, self.Ec,
                                     cfg.conv_k, _p(self.conv_y)), h)
                out_w, out_x = W[p + "shortconv.out_proj"], self.conv_y
            self._rowpar(h, out_w, out_x, self.o, f[p + "post_attention_norm"], f[p + "ffn_norm"])
            check(L.ef_gemv_swiglu(h, W[p + "ffn_gate"].h, W[p + "ffn_up"].h, _p(self.nrm), 1, _p(self.sw)), h)
            nxt = f[f"blk.{l + 1}.attn_norm"] if l + 1 < cfg.layers else f["output_norm"]
            self._rowpar(h, W[p + "ffn_down"], self.sw, self.d, f[p + "post_ffw_norm"], nxt)
        self._head(h, self.nrm)

    def _head(self, h, nrm_row: torch.Tensor):
        """Logits of the normalised row -> greedy token, position + 1, out_tokens."""
        L, cfg, W = self.L, self.cfg, self.w
        check(L.ef_gemv(h, W["output"].h, _p(nrm_row), 1, _p(self.logits)), h)
        if self.world == 1:
            check(L.ef_argmax_step(h, _p(self.logits), cfg.vocab, _p(self.tok), _p(self.pos), _p(self.out_tokens),
                                   self.out_base, cfg.max_pos), h)
        else:
            import torch.distributed as dist
            check(L.ef_argmax_partial(h, _p(self.logits), 1, self.Vl, self.rank * self.Vl, _p(self.pair)), h)
            if self.comm is not None:
                self.comm.all_gather(self.pairs, self.pair)
            else:
                dist.all_gather_into_tensor(self.pairs, self.pair)
            check(L.ef_argmax_select(h, _p(self.pairs), self.world, 1, _p(self.tok), _p(self.pos),
                                     _p(self.out_tokens), self.out_base, cfg.max_pos), h)

    def capture(self):
        """Record one step as a CUDA graph (after one eager step has sized every scratch)."""
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        self.graph = torch.cuda.CUDAGraph()
        # thread_local: the process group's watchdog thread may query events meanwhile
        with torch.cuda.graph(self.graph, stream=s, capture_error_mode="thread_local"):
            self.step()
        torch.cuda.synchronize()

    def run_step(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self.step()

    def prefill_steps(self, prompt: torch.Tensor):
        """Prompt ids one step each (the token each step predicts is replaced by
        the next prompt id); after the last one, self.tok is the first
        generated token."""
        prompt = prompt.to(self.tok.device, torch.int32)
        for i in range(prompt.numel()):
            self.tok.copy_(prompt[i:i + 1])
            self.run_step()

    def prefill(self, prompt: torch.Tensor):
        """All prompt ids at once, at positions pos .. pos + T - 1: every matrix
        product through the GEMM path (Q8_0 on tcgen05, f16 activations, the
        numerics of the GEMV), RoPE / cache / causal attention and the short
        convolution over the T tokens; then the head on the last row, so
        self.tok is the first generated token and pos has advanced by T (the
        reference's prompt forward, js/model.js:1135-1171)."""
        L, cfg, W, f = self.L, self.cfg, self.w, self.f32
        E, D, H, KV, Ec, Fl = cfg.hidden, cfg.head_dim, self.Hl, self.KVl, self.Ec, self.Fl
        T = int(prompt.numel())
        h = self.ops.ctx.bind()
        eps = ctypes.c_float(cfg.eps)
        dev = self.x.device
        z = lambda *s: torch.empty(*s, device=dev)
        x, nrm, o = z(T, E), z(T, E), z(T, E)
        q, k, v, g, att = z(T, H * D), z(T, KV * D), z(T, KV * D), z(T, H), z(T, H * D)
        bcx, cy, gt, up = z(T, 3 * Ec), z(T, Ec), z(T, Fl), z(T, Fl)
        ids = prompt.to(dev, torch.int32)
        gemm = lambda name, xin, out: check(L.ef_gemm(h, W[name].h, _p(xin), 0, T, _p(out), 0), h)

        def reduce(t):
            if self.world > 1:
                import torch.distributed as dist
                if self.comm is not None and self.comm.fits(t):
                    self.comm.all_reduce(t)
                else:
                    dist.all_reduce(t)

        check(L.ef_gather_rmsnorm(h, W["token_embd"].h, _p(ids), T, _p(f["blk.0.attn_norm"]), eps, _p(x), _p(nrm)), h)
        for l in range(cfg.layers):
            p = f"blk.{l}."
            if l in cfg.attn_layers:
                gemm(p + "attn_q", nrm, q)
                gemm(p + "attn_k", nrm, k)
                gemm(p + "attn_v", nrm, v)
                gemm(p + "attn_gate", nrm, g)
                check(self._rope(h, _p(q), _p(k), _p(v), _p(f[p + "attn_q_norm"]), _p(f[p + "attn_k_norm"]),
                                      _p(self.pos), 1, T, cfg.max_pos, H, KV, D, 2, ctypes.c_float(cfg.rope_theta),
                                      eps, _p(self.kc[l]), _p(self.vc[l])), h)
                check(self._attn(h, _p(q), _p(self.kc[l]), _p(self.vc[l]), _p(g), _p(self.pos), 1, T,
                                     cfg.max_pos, self.windows[l], H, KV, D, _p(att)), h)
                gemm(p + "attn_output", att, o)
            else:
                gemm(p + "shortconv.in_proj", nrm, bcx)
                check(L.ef_shortconv(h, _p(bcx), _p(f[p + "shortconv.conv"]), _p(self.state[l]), T, Ec, cfg.conv_k,
                                     _p(cy)), h)
                gemm(p + "shortconv.out_proj", cy, o)
            reduce(o)
            check(L.ef_norm_add_norm(h, _p(o), _p(f[p + "post_attention_norm"]), _p(x), _p(f[p + "ffn_norm"]), T, E,
                                     eps, _p(nrm)), h)
            gemm(p + "ffn_gate", nrm, gt)
            gemm(p + "ffn_up", nrm, up)
            check(L.ef_swiglu(h, _p(gt), _p(up), T * Fl, _p(gt)), h)
            gemm(p + "ffn_down", gt, o)
            reduce(o)
            nxt = f[f"blk.{l + 1}.attn_norm"] if l + 1 < cfg.layers else f["output_norm"]
            check(L.ef_norm_add_norm(h, _p(o), _p(f[p + "post_ffw_norm"]), _p(x), _p(nxt), T, E, eps, _p(nrm)), h)
        self.pos.add_(T - 1)                       # the head's step advances it to pos + T
        self._head(h, nrm[T - 1])

    def generate(self, prompt: torch.Tensor, n: int, use_graph: bool = True, batched_prompt: bool = True) -> list:
        """Greedy continuation of `prompt` by n tokens (the prompt all at once,
        or one step per id)."""
        self.reset(out_base=prompt.numel())
        # one eager step sizes the scratch and configures every kernel; then
        # the state is reset and the graph recorded
        self.tok.copy_(prompt[:1].to(self.tok.device, torch.int32))
        self.step()
        torch.cuda.synchronize()
        self.reset(out_base=prompt.numel())
        if batched_prompt:
            self.prefill(prompt)
            if use_graph:
                self.capture()
        else:
            if use_graph:
                self.capture()
            self.prefill_steps(prompt)
        for _ in range(n - 1):
            self.run_step()
        torch.cuda.synchronize()
        return self.out_tokens[:n].cpu().tolist()
