"""f32 -> GGUF block quantizers in torch (on any device), for the synthetic
model weights of the decoders (N(0, 0.02) tensors quantized from a seed).

The byte layouts are the ones the reference decodes (js/kernels.wgsl.js):
  Q8_0 (:153-169)  f16 d | 32 int8 q;                w = d * q
  Q4_K (:224-250)  f16 d | f16 dmin | 12 B of 6-bit (sc, m) x 8 packed as
                   scale_min_k4 (:94-104) | 128 B nibbles; sub-block j of 32
                   weights: w = d*sc_j*q - dmin*m_j
  Q6_K (:252-330)  ql[128] | qh[64] | int8 sc[16] | f16 d; sub-block j of 16
                   weights: w = d*sc_j*(q - 32)
The scale choices are plain ones (min/max per sub-block, no search): the
decoders only need valid blocks whose values follow the tensor.
"""
from __future__ import annotations

import torch


def _f16_bytes(v: torch.Tensor) -> torch.Tensor:
    """f32 [n] -> its f16 bits as uint8 [n][2] (little-endian)."""
    return v.to(torch.float16).view(torch.uint8).reshape(-1, 2)


def quantize_q8_0(w: torch.Tensor) -> torch.Tensor:
    """[rows][k] f32 -> Q8_0 bytes (uint8 1-D): d = max|x|/127 (f16), q =
    round-half-even(x / d) computed in f32."""
    b = w.reshape(-1, 32).float()
    d = b.abs().amax(dim=1) / 127.0
    inv = torch.where(d > 0, 1.0 / torch.where(d > 0, d, torch.ones_like(d)), torch.zeros_like(d))
    q = torch.clamp(torch.round(b * inv[:, None]), -127, 127).to(torch.int8)
    out = torch.empty(b.shape[0], 34, dtype=torch.uint8, device=w.device)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:] = q.view(torch.uint8)
    return out.reshape(-1)


def quantize_q4_k(w: torch.Tensor) -> torch.Tensor:
    """[rows][k] f32 (k a multiple of 256) -> Q4_K bytes. Per sub-block of 32:
    min m_j = min(0, min x), step s_j = (max x - m_j) / 15; per superblock d =
    max s_j / 63, dmin = max(-m_j) / 63 (both stored f16), sc_j = round(s_j/d),
    m_j' = round(-m_j/dmin) (6 bits), q = round((x + dmin*m_j') / (d*sc_j))
    clamped to [0, 15]."""
    x = w.reshape(-1, 8, 32).float()
    nb = x.shape[0]
    mn = torch.clamp(x.amin(dim=2), max=0.0)
    step = (x.amax(dim=2) - mn) / 15.0
    d = (step.amax(dim=1) / 63.0).to(torch.float16).float()
    dmin = ((-mn).amax(dim=1) / 63.0).to(torch.float16).float()
    safe = lambda v: torch.where(v > 0, v, torch.ones_like(v))
    sc = torch.where(d[:, None] > 0, torch.clamp(torch.round(step / safe(d)[:, None]), 0, 63), torch.zeros_like(step))
    m = torch.where(dmin[:, None] > 0, torch.clamp(torch.round(-mn / safe(dmin)[:, None]), 0, 63),
                    torch.zeros_like(mn))
    d1 = d[:, None] * sc
    m1 = dmin[:, None] * m
    q = torch.where(d1[..., None] > 0, torch.round((x + m1[..., None]) / safe(d1)[..., None]), torch.zeros_like(x))
    q = torch.clamp(q, 0, 15).to(torch.int32)                         # [nb][8][32]
    sc = sc.to(torch.int32)
    m = m.to(torch.int32)
    out = torch.empty(nb, 144, dtype=torch.uint8, device=w.device)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:4] = _f16_bytes(dmin)
    s = torch.empty(nb, 12, dtype=torch.int32, device=w.device)
    s[:, 0:4] = sc[:, 0:4] | ((sc[:, 4:8] >> 4) << 6)
    s[:, 4:8] = m[:, 0:4] | ((m[:, 4:8] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:8] & 0xF) | ((m[:, 4:8] & 0xF) << 4)
    out[:, 4:16] = s.to(torch.uint8)
    # byte 16 + 32j + l: low nibble = sub-block 2j, high nibble = sub-block 2j+1
    qs = q[:, 0::2, :] | (q[:, 1::2, :] << 4)                          # [nb][4][32]
    out[:, 16:] = qs.reshape(nb, 128).to(torch.uint8)
    return out.reshape(-1)


def quantize_q6_k(w: torch.Tensor) -> torch.Tensor:
    """[rows][k] f32 (k a multiple of 256) -> Q6_K bytes. Per sub-block of 16:
    s_j = max|x| / 32; per superblock d = max s_j / 127 (f16), sc_j =
    round(s_j / d) (int8), q = round(x / (d*sc_j)) clamped to [-32, 31], stored
    + 32."""
    x = w.reshape(-1, 16, 16).float()
    nb = x.shape[0]
    s = x.abs().amax(dim=2) / 32.0
    d = (s.amax(dim=1) / 127.0).to(torch.float16).float()
    safe = lambda v: torch.where(v != 0, v, torch.ones_like(v))
    sc = torch.where(d[:, None] > 0, torch.clamp(torch.round(s / safe(d)[:, None]), -128, 127), torch.zeros_like(s))
    ds = d[:, None] * sc
    q = torch.where(ds[..., None] != 0, torch.round(x / safe(ds)[..., None]), torch.zeros_like(x))
    q = (torch.clamp(q, -32, 31) + 32).to(torch.int32).reshape(nb, 2, 4, 32)   # [nb][half n][group g][l]
    ql = torch.empty(nb, 2, 64, dtype=torch.int32, device=w.device)
    ql[:, :, 0:32] = (q[:, :, 0] & 0xF) | ((q[:, :, 2] & 0xF) << 4)
    ql[:, :, 32:64] = (q[:, :, 1] & 0xF) | ((q[:, :, 3] & 0xF) << 4)
    qh = (q[:, :, 0] >> 4) | ((q[:, :, 1] >> 4) << 2) | ((q[:, :, 2] >> 4) << 4) | ((q[:, :, 3] >> 4) << 6)
    out = torch.empty(nb, 210, dtype=torch.uint8, device=w.device)
    out[:, 0:128] = ql.reshape(nb, 128).to(torch.uint8)
    out[:, 128:192] = qh.reshape(nb, 64).to(torch.uint8)
    out[:, 192:208] = sc.to(torch.int8).view(torch.uint8)
    out[:, 208:210] = _f16_bytes(d)
    return out.reshape(-1)


QUANTIZERS = {"Q8_0": quantize_q8_0, "Q4_K": quantize_q4_k, "Q6_K": quantize_q6_k}


def quantize(t: str, w: torch.Tensor) -> torch.Tensor:
    return QUANTIZERS[t](w)
