"""CPU restatement of the Llama-architecture decoder forward, for the
token-identity test of ``elffuss_engine_b200/llama.py``.

TEST INFRASTRUCTURE: only ``tests/`` use this module, as the checker; the
product never imports it.

It follows the reference's forward with the llama profile of js/state.js:
345-349: attnBlock (js/model.js:853-983) without QK-norm or gates, RoPE in
NORM pairing -- elements (2i, 2i+1) rotated by pos * base^(-2i/D)
(js/kernels.nn.wgsl.js:87-139, ROPE_NORM) --, causal grouped-query attention
with scale 1/sqrt(D) (softmaxShader :141-200), attn_output, then feedForward
(:635-664) without post-norms: x += o; SwiGLU on rmsnorm(x) * ffn_norm;
x += down. The head is `output` on rmsnorm(x) * output_norm (:1158-1171),
greedy with the lowest index winning ties (js/sample.js:95-99). Weights are
the exact dequantization (elffuss_oracle.c, pinned to the reference's
decoders by the golden vectors); all arithmetic in f64.

Tensor parallel (no counterpart in the reference): as in lfm3_ref.py, one
rank's shard with callbacks that sum over ranks and gather the argmax pairs.
Parity of this file with the reference's own code is unpinned (no model
tests in the reference, its CPU path cannot run here).
"""
from __future__ import annotations

import numpy as np

from . import dequant


def rmsnorm(x, w, eps):
    x = np.asarray(x, np.float64)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def rope_norm(x: np.ndarray, pos: int, base: float) -> np.ndarray:
    """x [heads][D]: pairs (2i, 2i+1) rotated by pos * base^(-2i/D)."""
    D = x.shape[-1]
    i = np.arange(D // 2)
    th = pos * base ** (-2.0 * i / D)
    c, s = np.cos(th), np.sin(th)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


class LlamaOracle:
    """cfg: an object with the LlamaConfig fields; weights: name -> (GGUF
    bytes, rows, k, type) or an f32 array (numpy)."""

    def __init__(self, cfg, weights: dict, rank: int = 0, world: int = 1, allreduce=None, allgather=None):
        self.cfg, self.rank, self.world = cfg, rank, world
        self.allreduce = allreduce or (lambda v: v)
        self.allgather = allgather
        self.w, self.f = {}, {}
        for name, val in weights.items():
            if isinstance(val, tuple):
                raw, rows, k, t = val
                self.w[name] = dequant(t, np.ascontiguousarray(raw)).reshape(rows, k).astype(np.float64)
            else:
                self.f[name] = np.asarray(val, np.float64)
        self.reset()

    def reset(self):
        self.kc = {l: [] for l in range(self.cfg.layers)}
        self.vc = {l: [] for l in range(self.cfg.layers)}
        self.pos = 0

    def logits(self, tok: int) -> np.ndarray:
        """Forward one token at self.pos; returns this rank's logits."""
        c, f, W = self.cfg, self.f, self.w
        D = c.head_dim
        H, KV = c.heads // self.world, c.kv_heads // self.world
        x = W["token_embd"][tok].copy()
        for l in range(c.layers):
            p = f"blk.{l}."
            nrm = rmsnorm(x, f[p + "attn_norm"], c.eps)
            q = rope_norm((W[p + "attn_q"] @ nrm).reshape(H, D), self.pos, c.rope_theta)
            k = rope_norm((W[p + "attn_k"] @ nrm).reshape(KV, D), self.pos, c.rope_theta)
            v = (W[p + "attn_v"] @ nrm).reshape(KV, D)
            self.kc[l].append(k)
            self.vc[l].append(v)
            K, V = np.stack(self.kc[l]), np.stack(self.vc[l])
            att = np.empty((H, D))
            for h in range(H):
                kvh = h // (H // KV)
                s = K[:, kvh, :] @ q[h] / np.sqrt(D)
                e = np.exp(s - s.max())
                att[h] = (e / e.sum()) @ V[:, kvh, :]
            x = x + self.allreduce(W[p + "attn_output"] @ att.reshape(-1))
            nrm = rmsnorm(x, f[p + "ffn_norm"], c.eps)
            g, u = W[p + "ffn_gate"] @ nrm, W[p + "ffn_up"] @ nrm
            x = x + self.allreduce(W[p + "ffn_down"] @ (g / (1.0 + np.exp(-g)) * u))
        self.pos += 1
        return W["output"] @ rmsnorm(x, f["output_norm"], c.eps)

    def step(self, tok: int) -> int:
        lg = self.logits(tok)
        i = int(np.argmax(lg))             # first maximum = lowest index wins ties
        if self.world == 1:
            return i
        pairs = self.allgather((float(lg[i]), i + self.rank * lg.size))
        best = max(v for v, _ in pairs)
        return min(ix for v, ix in pairs if v == best)

    def generate(self, prefix, last: int, n: int) -> list:
        """The prompt prefix + [last], then n greedy tokens."""
        self.reset()
        for t in prefix:
            self.logits(int(t))
        out = [self.step(int(last))]
        while len(out) < n:
            out.append(self.step(out[-1]))
        return out
