"""f32 restatement of the two decoder forwards, for the full-size token tests.

TEST INFRASTRUCTURE: only ``tests/`` use this module, as the checker of the
GPU decoders (``elffuss_engine_b200/lfm3.py`` and ``llama.py``); the product
never imports it.

Arithmetic: the reference GPU path's. Every weight is the exact f32
dequantisation of its GGUF blocks (``oracle.dequant``, the C restatement of
the reference decoders, js/kernels.wgsl.js:153-396,805-822), every activation
is f32, and every matrix product sums f32 products in f32, as the reference's
decode GEMV does (``d*q`` in f32 times f32 x, js/kernels.gemv.wgsl.js:247-276).
Unlike oracle/lfm3_ref.py (whose products use the f16 operands of the CUDA
kernels), nothing here rounds to f16 or quantises activations, so this
forward measures the CUDA path's distance from the reference's own numerics.

The code runs on torch tensors so that the 8B-shaped model (30 GB of f32
weights, a 4096-token context) can be evaluated on a GPU in seconds; torch's
TF32 modes are switched off while it runs, so its matrix products are f32
FMA chains like the reference's. On the CPU the same code runs unchanged.

The forwards follow the reference's js/model.js:
  * LFM3 (the lfm3 profile of js/state.js:345-349): convBlock :758-794
    (in_proj split B | C | x, B*x, causal depthwise conv over the previous
    kernel-1 inputs, C*y, out_proj), attnBlock :853-983 (per-head RMSNorm of q
    and k before NEOX RoPE, grouped-query attention with the causal and
    sliding-window mask of softmaxShader js/kernels.nn.wgsl.js:141-200, the
    head output times sigmoid(attn_gate(norm)), mulCabezaShader
    js/kernels.model.wgsl.js:89-105), feedForward :635-664 (post-norm,
    residual, FFN norm, SwiGLU, post-norm, residual), the tied head on the
    final norm (:1158-1171);
  * llama (the llama profile): no QK-norm, no gate, NORM RoPE pairing
    (2i, 2i+1), no post-norms: x += attn_output(att); x += ffn_down(SwiGLU(
    rmsnorm(x) * ffn_norm)); head `output` on rmsnorm(x) * output_norm.
RMSNorm is x / sqrt(mean(x^2) + eps) * w (kernels.nn.wgsl.js:46-80); RoPE
rotates pair i by pos * base^(-2i/D) (:87-139); greedy picks the first
maximum (js/sample.js:95-99). Parity with the reference's own code is
unpinned: the reference ships no model tests and its CPU path cannot run here.
"""
from __future__ import annotations

import contextlib

import numpy as np
import torch

from . import dequant


@contextlib.contextmanager
def strict_f32():
    """No TF32 in torch's f32 matrix products while the forward runs."""
    m, c = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = m, c


def _rmsnorm(x, w, eps):
    return x / torch.sqrt(torch.mean(x * x, dim=-1, keepdim=True) + eps) * w


def _rope(x, pos, base, neox: bool):
    """x [..., T, H, D] rotated at positions pos [T], angles in x's precision."""
    D = x.shape[-1]
    i = torch.arange(D // 2, device=x.device, dtype=x.dtype)
    th = pos.to(x.dtype)[:, None] * torch.pow(torch.tensor(base, dtype=x.dtype, device=x.device),
                                              -2.0 * i / D)[None, :]
    c, s = torch.cos(th)[:, None, :], torch.sin(th)[:, None, :]     # [T, 1, D/2]
    if neox:
        x0, x1 = x[..., :D // 2], x[..., D // 2:]
        return torch.cat([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def load_matrix(raw, rows: int, k: int, type_name: str, device, dtype=torch.float32) -> torch.Tensor:
    """Exact f32 dequantisation of one GGUF tensor (the C oracle, in row bands
    on host threads: the C call releases the GIL), on `device`."""
    from concurrent.futures import ThreadPoolExecutor
    b = np.ascontiguousarray(raw.cpu().numpy() if isinstance(raw, torch.Tensor) else raw, dtype=np.uint8)
    b = b.reshape(rows, -1)
    bands = [(r0, min(rows, r0 + 1024)) for r0 in range(0, rows, 1024)]
    with ThreadPoolExecutor(max_workers=16) as ex:
        parts = list(ex.map(lambda rr: dequant(type_name, b[rr[0]:rr[1]]).reshape(rr[1] - rr[0], k), bands))
    return torch.from_numpy(np.concatenate(parts, axis=0)).to(device, dtype)


class F32Decoder:
    """arch: "lfm3" or "llama"; cfg: LFM3Config / LlamaConfig fields; weights:
    name -> (GGUF bytes, rows, k[, type]) for matrices (LFM3 tuples carry no
    type: Q8_0) or f32 tensors. reset(1), forward(prompt ids [1][T]), then
    fork(S) gives S sequences that share that prompt, each with its own
    caches; forward(ids [S][1]) advances all of them by one token. dtype
    float64 runs the same forward in f64 (the CPU cross-check against the f64
    restatements)."""

    def __init__(self, arch: str, cfg, weights: dict, device="cpu", dtype=torch.float32):
        self.arch, self.cfg, self.dev, self.dt = arch, cfg, torch.device(device), dtype
        # f16 KV caches (cfg.kv_f16, the reference's kvF16: js/model.js:906-946,
        # kernels.attn.wgsl.js:51-55): k after its norm and RoPE and v are
        # rounded f32 -> f16 (to nearest even) when stored; all else unchanged
        self.kv16 = bool(getattr(cfg, "kv_f16", False))
        self.w, self.f = {}, {}
        for name, val in weights.items():
            if isinstance(val, tuple):
                raw, rows, k = val[:3]
                t = val[3] if len(val) > 3 else "Q8_0"
                self.w[name] = load_matrix(raw, rows, k, t, self.dev, dtype)
            else:
                self.f[name] = torch.as_tensor(val).to(self.dev, dtype)
        if arch == "lfm3":
            self.w["output"] = self.w["token_embd"]
            self.attn_layers = set(cfg.attn_layers)
            self.windows = cfg.windows()
        else:
            self.attn_layers = set(range(cfg.layers))
            self.windows = {l: 0 for l in range(cfg.layers)}

    # ---- state: per-layer caches [S][T][KV][D], conv states [S][K-1][E] ------
    def reset(self, S: int = 1):
        self.S, self.T = S, 0
        self.kc = {l: [] for l in self.attn_layers}
        self.vc = {l: [] for l in self.attn_layers}
        if self.arch == "lfm3":
            c = self.cfg
            self.conv = {l: torch.zeros(S, c.conv_k - 1, c.hidden, device=self.dev, dtype=self.dt)
                         for l in range(c.layers) if l not in self.attn_layers}

    def fork(self, S: int):
        """Copy sequence 0's state to S sequences (the batch shares its prompt)."""
        for d in (self.kc, self.vc):
            for l in d:
                d[l] = [t.expand(S, *t.shape[1:]).clone() for t in d[l]]
        if self.arch == "lfm3":
            for l in self.conv:
                self.conv[l] = self.conv[l].expand(S, *self.conv[l].shape[1:]).clone()
        self.S = S

    def _mm(self, name, x):
        return x @ self.w[name].T

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        """ids [S][T] at positions self.T .. self.T + T - 1 of each sequence;
        returns the logits [S][V] of the last position."""
        c, f = self.cfg, self.f
        S, T = ids.shape
        E, D, H, KV = c.hidden, c.head_dim, c.heads, c.kv_heads
        lfm = self.arch == "lfm3"
        pos = torch.arange(self.T, self.T + T, device=self.dev)
        with strict_f32():
            x = self.w["token_embd"][ids.to(self.dev).long()]                  # [S][T][E]
            nrm = _rmsnorm(x, f["blk.0.attn_norm"], c.eps)
            for l in range(c.layers):
                p = f"blk.{l}."
                if not lfm and l > 0:
                    nrm = _rmsnorm(x, f[p + "attn_norm"], c.eps)
                if l in self.attn_layers:
                    q = self._mm(p + "attn_q", nrm).view(S, T, H, D)
                    k = self._mm(p + "attn_k", nrm).view(S, T, KV, D)
                    v = self._mm(p + "attn_v", nrm).view(S, T, KV, D)
                    if lfm:
                        q = _rmsnorm(q, f[p + "attn_q_norm"], c.eps)
                        k = _rmsnorm(k, f[p + "attn_k_norm"], c.eps)
                    q, k = _rope(q, pos, c.rope_theta, lfm), _rope(k, pos, c.rope_theta, lfm)
                    if self.kv16:
                        k, v = k.float().half().to(self.dt), v.float().half().to(self.dt)
                    self.kc[l].append(k)
                    self.vc[l].append(v)
                    K = torch.cat(self.kc[l], dim=1)                             # [S][n][KV][D]
                    V = torch.cat(self.vc[l], dim=1)
                    n = K.shape[1]
                    keys = torch.arange(n, device=self.dev)
                    win = self.windows[l]
                    vis = keys[None, :] <= pos[:, None]
                    if win:
                        vis = vis & (pos[:, None] - keys[None, :] < win)
                    G = H // KV
                    qg = q.view(S, T, KV, G, D).permute(0, 2, 3, 1, 4)              # [S][KV][G][T][D]
                    Kt = K.permute(0, 2, 3, 1)                                      # [S][KV][D][n]
                    att = torch.empty(S, KV, G, T, D, device=self.dev, dtype=self.dt)
                    for t0 in range(0, T, 512):                                     # query blocks (memory)
                        sc = (qg[:, :, :, t0:t0 + 512] @ Kt[:, :, None]) / float(np.sqrt(D))
                        sc = sc.masked_fill(~vis[t0:t0 + 512][None, None, None], float("-inf"))
                        pr = torch.softmax(sc, dim=-1)
                        att[:, :, :, t0:t0 + 512] = pr @ V.permute(0, 2, 1, 3)[:, :, None]
                    att = att.permute(0, 3, 1, 2, 4).reshape(S, T, H, D)
                    if lfm:
                        g = self._mm(p + "attn_gate", nrm)                          # [S][T][H]
                        att = att / (1.0 + torch.exp(-g))[..., None]
                    o = self._mm(p + "attn_output", att.reshape(S, T, H * D))
                else:
                    bcx = self._mm(p + "shortconv.in_proj", nrm)
                    B, C, xs = bcx[..., :E], bcx[..., E:2 * E], bcx[..., 2 * E:]
                    bx = B * xs                                                     # [S][T][E]
                    w = f[p + "shortconv.conv"]                                     # [E][K], r = 0 oldest
                    seq = torch.cat([self.conv[l], bx], dim=1)                     # [S][K-1+T][E]
                    Kc = c.conv_k
                    conv = sum(seq[:, r:r + T] * w[:, r] for r in range(Kc))
                    o = self._mm(p + "shortconv.out_proj", C * conv)
                    self.conv[l] = seq[:, T:]
                if lfm:
                    x = x + _rmsnorm(o, f[p + "post_attention_norm"], c.eps)
                else:
                    x = x + o
                nrm = _rmsnorm(x, f[p + "ffn_norm"], c.eps)
                gate = self._mm(p + "ffn_gate", nrm)
                up = self._mm(p + "ffn_up", nrm)
                dn = self._mm(p + "ffn_down", gate / (1.0 + torch.exp(-gate)) * up)
                if lfm:
                    x = x + _rmsnorm(dn, f[p + "post_ffw_norm"], c.eps)
                    nxt = f[f"blk.{l + 1}.attn_norm"] if l + 1 < c.layers else f["output_norm"]
                    nrm = _rmsnorm(x, nxt, c.eps)
                else:
                    x = x + dn
            if not lfm:
                nrm = _rmsnorm(x, f["output_norm"], c.eps)
            logits = self._mm("output", nrm[:, -1])
        self.T += T
        return logits
