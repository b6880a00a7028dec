"""The f32 decoder forwards (oracle/forward_f32.py) on the CPU, run in f64
against the f64 restatements they must equal: oracle/lfm3_ref.py with exact
weights and oracle/llama_ref.py; batched prompts against one step per id; a
forked batch against separate sequences; f32 against f64 greedy tokens."""
import numpy as np
import torch

from elffuss_engine_b200.lfm3 import SMALL as LSMALL, LFM3Config, synth_weights as lfm3_weights
from elffuss_engine_b200.llama import SMALL as MSMALL, LlamaConfig, synth_weights as llama_weights
from oracle.forward_f32 import F32Decoder
from oracle.lfm3_ref import LFM3Oracle
from oracle.llama_ref import LlamaOracle


def _np(w):
    return {k: ((v[0].numpy(),) + tuple(v[1:]) if isinstance(v, tuple) else v.numpy()) for k, v in w.items()}


def test_lfm3_f64_equals_restatement_stepwise_and_batched():
    cfg = LFM3Config(**LSMALL)
    w = _np(lfm3_weights(cfg, seed=5))
    ids = np.random.default_rng(1).integers(0, cfg.vocab, 12)
    orc = LFM3Oracle(cfg, w, matmul="exact")
    want = []
    for t in ids:
        orc.step(int(t))
        want.append(orc.last_logits)
    dec = F32Decoder("lfm3", cfg, w, dtype=torch.float64)
    dec.reset(1)
    got = [dec.forward(torch.tensor([[int(t)]]))[0].numpy() for t in ids]
    scale = np.abs(np.stack(want)).max()
    assert np.max(np.abs(np.stack(got) - np.stack(want))) <= 1e-10 * scale
    dec.reset(1)
    batched = dec.forward(torch.tensor(ids[None, :8]))[0].numpy()
    assert np.max(np.abs(batched - want[7])) <= 1e-10 * scale
    for i in range(8, 12):                      # steps after a batched prompt
        assert np.max(np.abs(dec.forward(torch.tensor([[int(ids[i])]]))[0].numpy() - want[i])) <= 1e-10 * scale


def test_llama_f64_equals_restatement_and_fork():
    cfg = LlamaConfig(**MSMALL)
    w = _np(llama_weights(cfg, seed=6))
    ids = np.random.default_rng(2).integers(0, cfg.vocab, 14)
    prefix, lasts = ids[:10], [int(t) for t in ids[10:]]
    orc = LlamaOracle(cfg, w)
    want = []
    for last in lasts:
        orc.reset()
        for t in prefix:
            orc.logits(int(t))
        want.append(orc.logits(last))
    dec = F32Decoder("llama", cfg, w, dtype=torch.float64)
    dec.reset(1)
    dec.forward(torch.tensor(prefix[None, :]))
    dec.fork(len(lasts))
    got = dec.forward(torch.tensor(lasts)[:, None]).numpy()
    scale = np.abs(np.stack(want)).max()
    assert np.max(np.abs(got - np.stack(want))) <= 1e-10 * scale


def test_f32_tokens_equal_f64_tokens_small_models():
    for arch, cfg, w in (("lfm3", LFM3Config(**LSMALL), None), ("llama", LlamaConfig(**MSMALL), None)):
        w = _np(lfm3_weights(cfg, seed=7) if arch == "lfm3" else llama_weights(cfg, seed=7))
        ids = np.random.default_rng(3).integers(0, cfg.vocab, 9)
        toks = {}
        for dt in (torch.float32, torch.float64):
            dec = F32Decoder(arch, cfg, w, dtype=dt)
            dec.reset(1)
            lg = dec.forward(torch.tensor(ids[None, :]))
            out = []
            for _ in range(8):
                out.append(int(torch.argmax(lg[0])))
                lg = dec.forward(torch.tensor([[out[-1]]]))
            toks[dt] = out
        assert toks[torch.float32] == toks[torch.float64]


def test_f16_kv_cache_rounds_every_stored_entry():
    """cfg.kv_f16: the f32 forward keeps k and v in its caches as f16 values
    (round to nearest even from the f32 values); the logits stay close to the
    f32-cache forward's."""
    import dataclasses
    for arch, cfg in (("lfm3", LFM3Config(**LSMALL)), ("llama", LlamaConfig(**MSMALL))):
        w = _np(lfm3_weights(cfg, seed=7) if arch == "lfm3" else llama_weights(cfg, seed=7))
        ids = torch.tensor(np.random.default_rng(5).integers(0, cfg.vocab, 6)[None, :])
        out = {}
        for kv16 in (False, True):
            dec = F32Decoder(arch, dataclasses.replace(cfg, kv_f16=kv16), w)
            dec.reset(1)
            out[kv16] = dec.forward(ids)
            if kv16:
                for d in (dec.kc, dec.vc):
                    for ts in d.values():
                        t = torch.cat(ts, dim=1)
                        assert torch.equal(t, t.half().float())
        lo, lh = out[False][0].double(), out[True][0].double()
        assert float((lo - lh).abs().max()) < 0.05 * float(lo.std())
