"""CPU restatement of the LFM3 decoder forward, for the token-identity test.

TEST INFRASTRUCTURE: only ``tests/`` use this module, as the checker of the
GPU decoder in ``elffuss_engine_b200/lfm3.py``; the product never imports it.

It follows the reference's forward (js/model.js): convBlock :758-794 (in_proj
split B | C | x, B*x, causal depthwise conv over the window of the previous
kernel-1 values, C*y, out_proj), attnBlock :853-983 (per-head QK RMSNorm
before NEOX RoPE, grouped-query attention with causal + sliding-window mask
as in softmaxShader js/kernels.nn.wgsl.js:141-200, output times
sigmoid(attn_gate(norm)) per head as in mulCabezaShader
js/kernels.model.wgsl.js:89-105), feedForward :635-664 (post-norm, residual,
FFN norm, SwiGLU, post-norm, residual), the tied head on the final norm
(:1158-1171) and greedy argmax with the lowest index winning ties
(js/sample.js:95-99). RMSNorm is x / sqrt(mean(x^2) + eps) * w
(kernels.nn.wgsl.js:46-80); RoPE pairs (i, i + D/2) at angle
pos * base^(-2i/D) (:87-139); the embedding is the exact f32 dequant of the
Q8_0 row (quant.gather).

Arithmetic: f64 throughout, except that every matrix product takes its
operands at the precision of the f16 tensor-core GEMV it checks -- weights as
f16(d*q), activations rounded to f16 -- so that the remaining difference to
the GPU is f32 accumulation order, and greedy tokens can be compared exactly.
With matmul="f32" (for the full-size model, whose f64 weights would not fit
a test's memory) the products of those same f16 operands are summed in f32
by the host BLAS; everything else stays f64. With matmul="exact" the products
take the exact dequantised weights and unrounded activations, all f64 (the
cross-check of oracle/forward_f32.py).
Parity of this file with the reference's own code is unpinned: the reference
ships no model tests and its CPU path (Node + WebAssembly) cannot run here; it
is a restatement of the cited code.

Tensor parallel (no counterpart in the reference, which runs on one device):
given one rank's shard of the weights (lfm3.shard_weights) and callbacks that
sum a vector over the ranks and gather one (value, index) pair per rank, the
same forward runs on the local heads / channels / rows, so that the sharding
rules can be checked on the CPU against the unsharded forward.
"""
from __future__ import annotations

import numpy as np


def dequant_q8_0(raw: np.ndarray, rows: int, k: int) -> np.ndarray:
    """Exact f32 dequant d*q of Q8_0 bytes (kernels.wgsl.js:153-169)."""
    b = np.ascontiguousarray(raw, dtype=np.uint8).reshape(rows, k // 32, 34)
    d = b[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    q = b[..., 2:].copy().view(np.int8).astype(np.float32)
    return (d[..., None] * q).reshape(rows, k)


def f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, np.float64).astype(np.float16).astype(np.float64)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.asarray(x, np.float64)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def rope_neox(x: np.ndarray, pos: int, base: float) -> np.ndarray:
    """x [heads][D]: pairs (i, i + D/2) rotated by pos * base^(-2i/D)."""
    D = x.shape[-1]
    i = np.arange(D // 2)
    th = pos * base ** (-2.0 * i / D)
    c, s = np.cos(th), np.sin(th)
    x0, x1 = x[..., :D // 2], x[..., D // 2:]
    return np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1)


class LFM3Oracle:
    """cfg: an object with the LFM3Config fields; weights: name -> (Q8_0 bytes,
    rows, k) or an f32 array (numpy)."""

    def __init__(self, cfg, weights: dict, rank: int = 0, world: int = 1, allreduce=None, allgather=None,
                 matmul: str = "f64"):
        self.cfg = cfg
        self.f32 = matmul == "f32"
        self.exact = matmul == "exact"
        self.rank, self.world = rank, world
        self.allreduce = allreduce or (lambda v: v)
        self.allgather = allgather
        self.w16, self.f = {}, {}
        for name, val in weights.items():
            if isinstance(val, tuple):
                raw, rows, k = val
                w = dequant_q8_0(raw, rows, k)
                if self.exact:
                    self.w16[name] = w.astype(np.float64)
                else:
                    self.w16[name] = w.astype(np.float16).astype(np.float32 if self.f32 else np.float64)
                if name == "token_embd":
                    self.embd = w if self.f32 else w.astype(np.float64)
            else:
                self.f[name] = np.asarray(val, np.float64)
        self.windows = cfg.windows()
        self.reset()

    def reset(self):
        c = self.cfg
        ec = c.hidden // self.world
        self.state = {l: np.zeros((c.conv_k - 1, ec)) for l in range(c.layers) if l not in c.attn_layers}
        self.kc = {l: [] for l in c.attn_layers}
        self.vc = {l: [] for l in c.attn_layers}
        self.pos = 0

    def mm(self, name: str, x: np.ndarray) -> np.ndarray:
        if self.exact:
            return self.w16[name] @ np.asarray(x, np.float64)
        if self.f32:
            return (self.w16[name] @ f16(x).astype(np.float32)).astype(np.float64)
        return self.w16[name] @ f16(x)

    def step(self, tok: int) -> int:
        c, f = self.cfg, self.f
        E, D = c.hidden, c.head_dim
        H, KV, Ec = c.heads // self.world, c.kv_heads // self.world, c.hidden // self.world
        x = self.embd[tok].astype(np.float64)
        nrm = rmsnorm(x, f["blk.0.attn_norm"], c.eps)
        for l in range(c.layers):
            p = f"blk.{l}."
            if l in c.attn_layers:
                q = self.mm(p + "attn_q", nrm).reshape(H, D)
                k = self.mm(p + "attn_k", nrm).reshape(KV, D)
                v = self.mm(p + "attn_v", nrm).reshape(KV, D)
                g = self.mm(p + "attn_gate", nrm)
                q = rope_neox(rmsnorm(q, f[p + "attn_q_norm"], c.eps), self.pos, c.rope_theta)
                k = rope_neox(rmsnorm(k, f[p + "attn_k_norm"], c.eps), self.pos, c.rope_theta)
                self.kc[l].append(k)
                self.vc[l].append(v)
                K = np.stack(self.kc[l])          # [n][KV][D]
                V = np.stack(self.vc[l])
                n = K.shape[0]
                win = self.windows[l]
                keys = np.arange(n)
                vis = (keys <= self.pos) & ((win == 0) | (self.pos - keys < win))
                att = np.empty((H, D))
                for h in range(H):
                    kvh = h // (H // KV)
                    s = K[:, kvh, :] @ q[h] / np.sqrt(D)
                    s = np.where(vis, s, -np.inf)
                    e = np.exp(s - s.max())
                    pr = e / e.sum()
                    att[h] = (pr @ V[:, kvh, :]) / (1.0 + np.exp(-g[h]))
                o = self.mm(p + "attn_output", att.reshape(-1))
            else:
                bcx = self.mm(p + "shortconv.in_proj", nrm)
                B, C, xs = bcx[:Ec], bcx[Ec:2 * Ec], bcx[2 * Ec:]
                bx = B * xs
                st = self.state[l]
                w = f[p + "shortconv.conv"]                   # [E][K], r = 0 oldest
                win = np.concatenate([st, bx[None, :]], axis=0)  # [K][E]
                conv = np.sum(win.T * w, axis=1)
                y = C * conv
                self.state[l] = win[1:]
                o = self.mm(p + "shortconv.out_proj", y)
            o = self.allreduce(o)
            x = x + rmsnorm(o, f[p + "post_attention_norm"], c.eps)
            nrm = rmsnorm(x, f[p + "ffn_norm"], c.eps)
            gate = self.mm(p + "ffn_gate", nrm)
            up = self.mm(p + "ffn_up", nrm)
            sw = gate / (1.0 + np.exp(-gate)) * up
            dn = self.allreduce(self.mm(p + "ffn_down", sw))
            x = x + rmsnorm(dn, f[p + "post_ffw_norm"], c.eps)
            nxt = f[f"blk.{l + 1}.attn_norm"] if l + 1 < c.layers else f["output_norm"]
            nrm = rmsnorm(x, nxt, c.eps)
        self.pos += 1
        if self.world == 1:
            logits = self.mm("token_embd", nrm)
            self.last_logits = logits
            return int(np.argmax(logits))     # first maximum = lowest index wins ties
        logits = self.mm("output", nrm)       # this rank's vocabulary rows
        i = int(np.argmax(logits))
        pairs = self.allgather((float(logits[i]), i + self.rank * logits.size))
        best = max(v for v, _ in pairs)
        return min(ix for v, ix in pairs if v == best)

    def generate(self, prompt, n: int) -> list:
        self.reset()
        out = []
        tok = None
        for t in prompt:
            tok = self.step(int(t))
        out.append(tok)
        while len(out) < n:
            tok = self.step(tok)
            out.append(tok)
        return out
