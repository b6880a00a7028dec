"""The LFM3 decoder restatement (oracle/lfm3_ref.py) on the CPU: shapes of the
benchmark configuration, the pieces against direct formulas, determinism."""
import numpy as np
import torch

from elffuss_engine_b200.lfm3 import SMALL, LFM3Config, quantize_q8_0_torch, synth_weights
from elffuss_engine_b200 import formats
from oracle.lfm3_ref import LFM3Oracle, dequant_q8_0, rmsnorm, rope_neox


def _np_weights(w):
    return {k: ((v[0].numpy(), v[1], v[2]) if isinstance(v, tuple) else v.numpy()) for k, v in w.items()}


def test_config3_weight_count():
    # hidden 2048, 16 layers (10 short-conv, 6 attention), FFN 8192, vocab 65536
    cfg = LFM3Config()
    assert len(cfg.attn_layers) == 6 and cfg.layers == 16
    assert cfg.weight_params() == 1_170_604_032
    assert cfg.weight_params() * 34 // 32 == 1_243_766_784


def test_torch_quantizer_matches_numpy():
    w = torch.randn(64, 256, generator=torch.Generator().manual_seed(3)) * 0.02
    a = quantize_q8_0_torch(w).numpy()
    b = formats.quantize_q8_0(w.numpy())
    assert np.array_equal(a, b)
    back = dequant_q8_0(a, 64, 256)
    assert np.max(np.abs(back - w.numpy())) <= 0.5 * np.abs(w.numpy()).max() / 127 * 1.01


def test_rmsnorm_and_rope():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 64))
    y = rmsnorm(x, np.ones(64), 1e-5)
    assert np.allclose(np.mean(y * y, axis=1), 1.0, atol=1e-4)
    r = rope_neox(y, 7, 1e6)
    assert np.allclose(np.linalg.norm(r, axis=1), np.linalg.norm(y, axis=1))   # a rotation
    assert np.allclose(rope_neox(y, 0, 1e6), y)


def test_oracle_small_decode_is_deterministic():
    cfg = LFM3Config(**SMALL)
    w = _np_weights(synth_weights(cfg, seed=1))
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, 12)
    a = LFM3Oracle(cfg, w).generate(prompt, 8)
    b = LFM3Oracle(cfg, w).generate(prompt, 8)
    assert a == b and len(a) == 8 and all(0 <= t < cfg.vocab for t in a)
