"""North-star acceptance at the full config-3 shape: the synthetic
LFM3-shaped decoder (hidden 2048, 16 layers, vocab 65536; the bench's seeded
weights) produces, for a 16-id prompt, the same first 32 greedy tokens as the
CPU restatement of the forward (oracle/lfm3_ref.py, its products of the same
f16 operands summed in f32 by the host BLAS)."""
import numpy as np
import pytest
import torch

from elffuss_engine_b200.lfm3 import LFM3Config, LFM3Decoder, synth_weights
from oracle.lfm3_ref import LFM3Oracle

pytestmark = pytest.mark.gpu


def test_config3_first_32_tokens_match_cpu_forward(ops):
    cfg = LFM3Config()
    w = synth_weights(cfg, seed=0, device="cuda")
    prompt = torch.tensor(np.random.default_rng(2).integers(0, cfg.vocab, 16), dtype=torch.int32)
    dec = LFM3Decoder(ops, cfg, w)
    got = dec.generate(prompt, 32)
    dec.graph = None
    del dec
    wc = {k: ((v[0].cpu().numpy(), v[1], v[2]) if isinstance(v, tuple) else v.cpu().numpy()) for k, v in w.items()}
    del w
    torch.cuda.empty_cache()
    want = LFM3Oracle(cfg, wc, matmul="f32").generate(prompt.numpy(), 32)
    assert got == want
