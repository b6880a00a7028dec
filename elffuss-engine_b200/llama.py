"""Synthetic Llama-architecture decoder (8B shape, Q4_K_M-style mix) driven
through the quantized GEMV / GEMM path, batch 1..16.

The reference runs llama in js/model.js with the profile of js/state.js:
345-349 (no QK-norm, no gate, NORM RoPE pairing (2i, 2i+1), pre-FFN norm
`ffn_norm`, no post-norms): per layer attn_norm, q/k/v projections, RoPE, k
and v into the cache, causal grouped-query attention, attn_output, residual,
ffn_norm, SwiGLU FFN, residual (attnBlock :853-983, feedForward :635-664); the
head is `output` on the final norm of the last token (:1158-1171), greedy
(js/sample.js:95-99).

Weights: N(0, 0.02) quantized from a seed, Q4_K everywhere except Q6_K for
attn_v, for ffn_down of even layers and for the output head (the llama.cpp
Q4_K_M recipe); token_embd Q4_K; norms 1.

Work: a prompt's tokens go through the GEMM path (ef_gemm, all tokens of a
layer per call) with one causal attention call over the whole prompt; a decode
step runs B sequences at once (one token each) through the GEMV path (M = B)
and is captured as a CUDA graph. A batch of B distinct sequences is made from
one prompt: its first T-1 tokens are computed once and their caches copied to
every sequence, whose last prompt token differs.

Tensor parallel as in lfm3.py: q/k/v by heads, ffn_gate/up by inner rows,
output by vocabulary rows (column-parallel); attn_output and ffn_down by
input columns, each followed by an all-reduce (row-parallel); a local argmax
per rank, then the ranks' (value, index) pairs pick the token.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import formats
from ._lib import check, lib
from .quantize import quantize

EF_F32 = 0
ROPE_NORM = 0


@dataclass
class LlamaConfig:
    hidden: int = 4096
    layers: int = 32
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rope_theta: float = 5e5
    eps: float = 1e-5
    max_pos: int = 4096 + 256     # KV-cache capacity per sequence
    kv_f16: bool = False          # f16 KV caches (the reference's kvF16 option), f32 by default

    def weight_type(self, name: str) -> str:
        short = name.split(".", 2)[-1] if name.startswith("blk.") else name
        if short == "attn_v" or name == "output":
            return "Q6_K"
        if short == "ffn_down" and int(name.split(".")[1]) % 2 == 0:
            return "Q6_K"
        return "Q4_K"

    def matrices(self):
        """(name, rows, k) of every quantized tensor."""
        E, H, KV, D, F = self.hidden, self.heads, self.kv_heads, self.head_dim, self.ffn
        out = [("token_embd", self.vocab, E), ("output", self.vocab, E)]
        for l in range(self.layers):
            p = f"blk.{l}."
            out += [(p + "attn_q", H * D, E), (p + "attn_k", KV * D, E), (p + "attn_v", KV * D, E),
                    (p + "attn_output", E, H * D), (p + "ffn_gate", F, E), (p + "ffn_up", F, E),
                    (p + "ffn_down", E, F)]
        return out

    def step_weight_bytes(self) -> int:
        """Bytes of the weights one decode step reads (all but token_embd)."""
        return sum(formats.tensor_bytes(self.weight_type(n), r, k) for n, r, k in self.matrices()
                   if n != "token_embd")


SMALL = dict(hidden=512, layers=2, heads=4, kv_heads=2, head_dim=128, ffn=768, vocab=1024, max_pos=96)


def synth_weights(cfg: LlamaConfig, seed: int = 0, device: str = "cpu") -> dict:
    """name -> (GGUF bytes (uint8 1-D), rows, k, type) for the matrices, f32
    tensors for the norms. Matrix i draws N(0, 0.02) from a generator seeded
    with seed * 1000 + i on `device`, in row bands of at most 2^26 values."""
    out = {}
    for i, (name, rows, k) in enumerate(cfg.matrices()):
        t = cfg.weight_type(name)
        g = torch.Generator(device=device)
        g.manual_seed(seed * 1000 + i)
        band = max(1, (1 << 26) // k)
        parts = []
        for r0 in range(0, rows, band):
            n = min(band, rows - r0)
            parts.append(quantize(t, torch.empty(n, k, device=device).normal_(0.0, 0.02, generator=g)))
        out[name] = (torch.cat(parts), rows, k, t)
    ones = lambda n: torch.ones(n, device=device)
    out["output_norm"] = ones(cfg.hidden)
    for l in range(cfg.layers):
        out[f"blk.{l}.attn_norm"] = ones(cfg.hidden)
        out[f"blk.{l}.ffn_norm"] = ones(cfg.hidden)
    return out


def _rows(raw, t, rows, k, r0, r1):
    be, bb = formats.block_info(t)
    return raw.reshape(rows, (k // be) * bb)[r0:r1].reshape(-1).contiguous()


def _cols(raw, t, rows, k, c0, c1):
    be, bb = formats.block_info(t)
    return raw.reshape(rows, k // be, bb)[:, c0 // be:c1 // be].reshape(-1).contiguous()


def shard_weights(cfg: LlamaConfig, weights: dict, rank: int, world: int) -> dict:
    """Rank `rank` of `world`'s slices (module docstring); token_embd whole."""
    E, H, KV, D, F, V = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab
    g, r = world, rank
    for what, n in (("heads", H), ("kv_heads", KV), ("ffn", F), ("vocab", V)):
        if n % g:
            raise ValueError(f"tensor parallel over {g} ranks: {what}={n} does not split")
    Hl, KVl, Fl, Vl = H // g, KV // g, F // g, V // g
    for what, n in (("heads*head_dim", Hl * D), ("ffn", Fl)):
        if n % 256:
            raise ValueError(f"tensor parallel over {g} ranks: the {what} slice {n} is not a multiple of 256")
    out = {}
    for name, val in weights.items():
        if not isinstance(val, tuple):
            out[name] = val
            continue
        raw, rows, k, t = val
        short = name.split(".", 2)[-1] if name.startswith("blk.") else name
        if short == "token_embd":
            out[name] = val
        elif short == "output":
            out[name] = (_rows(raw, t, rows, k, r * Vl, (r + 1) * Vl), Vl, k, t)
        elif short == "attn_q":
            out[name] = (_rows(raw, t, rows, k, r * Hl * D, (r + 1) * Hl * D), Hl * D, k, t)
        elif short in ("attn_k", "attn_v"):
            out[name] = (_rows(raw, t, rows, k, r * KVl * D, (r + 1) * KVl * D), KVl * D, k, t)
        elif short == "attn_output":
            out[name] = (_cols(raw, t, rows, k, r * Hl * D, (r + 1) * Hl * D), rows, Hl * D, t)
        elif short in ("ffn_gate", "ffn_up"):
            out[name] = (_rows(raw, t, rows, k, r * Fl, (r + 1) * Fl), Fl, k, t)
        elif short == "ffn_down":
            out[name] = (_cols(raw, t, rows, k, r * Fl, (r + 1) * Fl), rows, Fl, t)
        else:
            raise ValueError(f"no shard rule for {name}")
    return out


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _pp(ts):
    arr = (ctypes.c_void_p * len(ts))(*[t if isinstance(t, int) else t.data_ptr() for t in ts])
    return ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p))


class LlamaDecoder:
    """B sequences decoded together (see the module docstring). With
    world > 1, `weights` are this rank's shard_weights and the collectives go
    through torch.distributed's default (NCCL) process group."""

    def __init__(self, ops, cfg: LlamaConfig, weights: dict, batch: int = 1, rank: int = 0, world: int = 1,
                 pdl: bool = True, out_cap: int = 512, comm=None, fused: bool = True):
        if not 1 <= batch <= 16:
            raise ValueError("batch must be 1..16 (the GEMV path)")
        self.ops, self.cfg, self.L = ops, cfg, lib()
        self.B, self.rank, self.world, self.pdl, self.out_cap = batch, rank, world, pdl, out_cap
        self.comm, self.fused = comm, fused
        E, D = cfg.hidden, cfg.head_dim
        self.Hl, self.KVl, self.Fl, self.Vl = cfg.heads // world, cfg.kv_heads // world, cfg.ffn // world, \
            cfg.vocab // world
        self.dev = dev = torch.device("cuda", ops.ctx.device)
        self.w, self.f32 = {}, {}
        for name, val in weights.items():
            if isinstance(val, tuple):
                raw, rows, k, t = val
                self.w[name] = ops.load_weight(t, raw.to(dev), rows, k, label=name)
            else:
                self.f32[name] = val.to(dev).float().contiguous()
        B, Hl, KVl = batch, self.Hl, self.KVl
        z = lambda *s: torch.zeros(*s, device=dev)
        self.x, self.nrm, self.o, self.d = z(B, E), z(B, E), z(B, E), z(B, E)
        self.q, self.k, self.v, self.att = z(B, Hl * D), z(B, KVl * D), z(B, KVl * D), z(B, Hl * D)
        self.sw = z(B, self.Fl)
        self.logits = z(B, self.Vl)
        self.pairs1 = torch.zeros(B, 2, dtype=torch.int32, device=dev)
        self.pairs = torch.zeros(world * B * 2, dtype=torch.int32, device=dev)
        kvt = torch.float16 if cfg.kv_f16 else torch.float32
        self.kc = [torch.zeros(B, cfg.max_pos, KVl, D, dtype=kvt, device=dev) for _ in range(cfg.layers)]
        self.vc = [torch.zeros(B, cfg.max_pos, KVl, D, dtype=kvt, device=dev) for _ in range(cfg.layers)]
        sfx = "_f16" if cfg.kv_f16 else ""
        self._rope = getattr(self.L, "ef_rope_cache" + sfx)
        self._attn = getattr(self.L, "ef_attention" + sfx)
        self.tok = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.out_tokens = torch.full((B, out_cap), -1, dtype=torch.int32, device=dev)
        self.out_base = 0
        self.graph = None

    # -- helpers ---------------------------------------------------------------
    def _reduce(self, t):
        """In-place sum over the ranks: the peer-memory collectives (tp.TPComm)
        when given and the data fits them, else NCCL."""
        if self.world > 1:
            if self.comm is not None:
                self.comm.all_reduce(t)
            else:
                import torch.distributed as dist
                dist.all_reduce(t)

    def _rowpar(self, h, w, xin, out, w_next):
        """out = w xin for the B rows (this rank's columns), summed over the
        ranks; then x += out and nrm = rmsnorm(x) * w_next. With the
        peer-memory collectives, one fused call (ef_gemv_allreduce_norm)."""
        L, eps = self.L, ctypes.c_float(self.cfg.eps)
        if self.world > 1 and self.comm is not None and self.fused:
            check(L.ef_gemv_allreduce_norm(h, self.comm.tp, w.h, _p(xin), self.B, None, _p(self.x), _p(w_next),
                                           eps, _p(self.nrm)), h)
            return
        check(L.ef_gemv(h, w.h, _p(xin), self.B, _p(out)), h)
        self._reduce(out)
        check(L.ef_norm_add_norm(h, _p(out), None, _p(self.x), _p(w_next), self.B, self.cfg.hidden, eps,
                                 _p(self.nrm)), h)

    def _head(self, h, rows):
        """logits of `rows` rows of self.nrm -> tokens / positions / out_tokens."""
        L, cfg = self.L, self.cfg
        check(L.ef_gemv(h, self.w["output"].h, _p(self.nrm), rows, _p(self.logits)), h)
        if self.world == 1:
            check(L.ef_argmax_rows(h, _p(self.logits), rows, self.Vl, _p(self.tok), _p(self.pos),
                                   _p(self.out_tokens), self.out_base, self.out_cap), h)
        else:
            import torch.distributed as dist
            check(L.ef_argmax_partial(h, _p(self.logits), rows, self.Vl, self.rank * self.Vl, _p(self.pairs1)), h)
            if self.comm is not None:
                self.comm.all_gather(self.pairs, self.pairs1.view(-1))
            else:
                dist.all_gather_into_tensor(self.pairs, self.pairs1.view(-1))
            check(L.ef_argmax_select(h, _p(self.pairs), self.world, rows, _p(self.tok), _p(self.pos),
                                     _p(self.out_tokens), self.out_base, self.out_cap), h)

    # -- one decode step: a token for each of the B sequences ------------------
    def step(self):
        L, h = self.L, self.ops.ctx.bind()
        check(L.ef_ctx_set_pdl(h, 1 if self.pdl else 0), h)
        try:
            self._step(h)
        finally:
            L.ef_ctx_set_pdl(h, 1)   # the context default

    def _step(self, h):
        L, cfg, W, f = self.L, self.cfg, self.w, self.f32
        B, E, D = self.B, cfg.hidden, cfg.head_dim
        eps = ctypes.c_float(cfg.eps)
        check(L.ef_gather_rmsnorm(h, W["token_embd"].h, _p(self.tok), B, _p(f["blk.0.attn_norm"]), eps, _p(self.x),
                                  _p(self.nrm)), h)
        for l in range(cfg.layers):
            p = f"blk.{l}."
            check(L.ef_gemv_sections(h, _pp([W[p + "attn_q"].h.value, W[p + "attn_k"].h.value]), 2, _p(self.nrm),
                                     B, _pp([self.q, self.k])), h)
            check(L.ef_gemv(h, W[p + "attn_v"].h, _p(self.nrm), B, _p(self.v)), h)
            check(self._rope(h, _p(self.q), _p(self.k), _p(self.v), None, None, _p(self.pos), B, 1,
                                  cfg.max_pos, self.Hl, self.KVl, D, ROPE_NORM, ctypes.c_float(cfg.rope_theta), eps,
                                  _p(self.kc[l]), _p(self.vc[l])), h)
            check(self._attn(h, _p(self.q), _p(self.kc[l]), _p(self.vc[l]), None, _p(self.pos), B, 1,
                                 cfg.max_pos, 0, self.Hl, self.KVl, D, _p(self.att)), h)
            self._rowpar(h, W[p + "attn_output"], self.att, self.o, f[p + "ffn_norm"])
            check(L.ef_gemv_swiglu(h, W[p + "ffn_gate"].h, W[p + "ffn_up"].h, _p(self.nrm), B, _p(self.sw)), h)
            nxt = f[f"blk.{l + 1}.attn_norm"] if l + 1 < cfg.layers else f["output_norm"]
            self._rowpar(h, W[p + "ffn_down"], self.sw, self.d, nxt)
        self._head(h, B)

    def capture(self):
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s, capture_error_mode="thread_local"):
            self.step()
        torch.cuda.synchronize(self.dev)

    def run_step(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self.step()

    # -- prompt ----------------------------------------------------------------
    def prefill(self, ids: torch.Tensor):
        """The prompt's tokens ids (a 1-D int tensor) at positions 0..T-1 of
        sequence 0, all at once through the GEMM path; their k and v are in
        sequence 0's caches afterwards. No head (the next token comes from a
        step)."""
        L, cfg, W, f = self.L, self.cfg, self.w, self.f32
        E, D, T = cfg.hidden, cfg.head_dim, int(ids.numel())
        if T < 1 or T > cfg.max_pos:
            raise ValueError("prompt length outside the caches")
        h = self.ops.ctx.bind()
        eps = ctypes.c_float(cfg.eps)
        z = lambda *s: torch.empty(*s, device=self.dev)
        x, nrm, o = z(T, E), z(T, E), z(T, E)
        q, k, v, att = z(T, self.Hl * D), z(T, self.KVl * D), z(T, self.KVl * D), z(T, self.Hl * D)
        gt, up = z(T, self.Fl), z(T, self.Fl)
        ids_d = ids.to(self.dev, torch.int32)
        pos0 = torch.zeros(1, dtype=torch.int32, device=self.dev)
        gemm = lambda name, xin, out: check(L.ef_gemm(h, W[name].h, _p(xin), EF_F32, T, _p(out), 0), h)
        check(L.ef_gather_rmsnorm(h, W["token_embd"].h, _p(ids_d), T, _p(f["blk.0.attn_norm"]), eps, _p(x),
                                  _p(nrm)), h)
        for l in range(cfg.layers):
            p = f"blk.{l}."
            gemm(p + "attn_q", nrm, q)
            gemm(p + "attn_k", nrm, k)
            gemm(p + "attn_v", nrm, v)
            check(self._rope(h, _p(q), _p(k), _p(v), None, None, _p(pos0), 1, T, cfg.max_pos, self.Hl,
                                  self.KVl, D, ROPE_NORM, ctypes.c_float(cfg.rope_theta), eps, _p(self.kc[l]),
                                  _p(self.vc[l])), h)
            check(self._attn(h, _p(q), _p(self.kc[l]), _p(self.vc[l]), None, _p(pos0), 1, T, cfg.max_pos, 0,
                                 self.Hl, self.KVl, D, _p(att)), h)
            gemm(p + "attn_output", att, o)
            self._reduce(o)
            check(L.ef_norm_add_norm(h, _p(o), None, _p(x), _p(f[p + "ffn_norm"]), T, E, eps, _p(nrm)), h)
            gemm(p + "ffn_gate", nrm, gt)
            gemm(p + "ffn_up", nrm, up)
            check(L.ef_swiglu(h, _p(gt), _p(up), T * self.Fl, _p(gt)), h)
            gemm(p + "ffn_down", gt, o)
            self._reduce(o)
            nxt = f[f"blk.{l + 1}.attn_norm"] if l + 1 < cfg.layers else f["output_norm"]
            check(L.ef_norm_add_norm(h, _p(o), None, _p(x), _p(nxt), T, E, eps, _p(nrm)), h)

    def start(self, prompt: torch.Tensor, last_ids, out_base: int | None = None):
        """Sequences b = 0..B-1 with the prompt prompt[:-1] + [last_ids[b]]: the
        shared part once (prefill), its caches copied to every sequence; tok =
        last_ids, pos = T - 1, so the next step reads the last tokens and
        produces each sequence's first new token (out_tokens[b][0])."""
        T = int(prompt.numel())
        self.graph = None
        for c in self.kc + self.vc:
            c.zero_()
        self.prefill(prompt[:T - 1])
        for c in self.kc + self.vc:
            c[1:, :T - 1].copy_(c[0:1, :T - 1].expand(self.B - 1, -1, -1, -1))
        self.rewind(T, last_ids, out_base)

    def rewind(self, T: int, last_ids, out_base: int | None = None):
        """Back to the state right after start(): the caches up to position T-2
        are kept (a step writes position pos onwards), tok / pos / out_tokens
        are set again."""
        self.tok.copy_(torch.as_tensor(last_ids, dtype=torch.int32).to(self.dev))
        self.pos.fill_(T - 1)
        self.out_tokens.fill_(-1)
        self.out_base = T if out_base is None else out_base

    def generate(self, prompt: torch.Tensor, last_ids, n: int, use_graph: bool = True) -> list:
        """n greedy tokens for each of the B sequences (a list of B lists)."""
        T = int(prompt.numel())
        # one eager step sizes every scratch and configures every kernel; then
        # rewind and record the graph
        self.start(prompt, last_ids)
        self.step()
        torch.cuda.synchronize(self.dev)
        self.rewind(T, last_ids)
        if use_graph:
            self.capture()
        for _ in range(n):
            self.run_step()
        torch.cuda.synchronize(self.dev)
        return self.out_tokens[:, :n].cpu().tolist()
