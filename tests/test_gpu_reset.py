"""Segment-reset context (context_mode="reset") against the torch oracle:
after every boundary (and its update) the context is rebuilt from the last
block_size symbols at positions 0.., as the reference engine does."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from altxs_b200 import codec as C
from altxs_b200.config import ModelConfig
from oracle.model import OracleModel, OracleTTT, OracleWeights

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL = 2e-3

SMALL = dict(
    vocab_size=512, num_layers=3, model_dim=128, num_heads=4, num_kv_heads=2,
    mlp_mult=4.0, rope_dims=16, block_size=32, online_retrain_every=64, seed=11,
    ttt_lora_rank=4, ttt_lora_lr=1e-3, ttt_k_lora=True, ttt_o_lora=True, context_mode="reset",
)


def _motif_cfg_weights():
    """Every motif on (with a depth loop and parallel lanes), q/k/v/o/MLP adapters."""
    from tests.test_gpu_lora_motifs import _cfg, _weights

    cfg = _cfg("all", context_mode="reset", ttt_lora_rank=4, ttt_lora_lr=1e-3)
    return cfg, _weights(cfg, seed=21)


@pytest.mark.parametrize("tensor_cores", [True, False])
@pytest.mark.parametrize("with_updates", [False, True])
def test_reset_with_motifs_matches_oracle(with_updates, tensor_cores):
    """The reset prefill on a motif model (one K/V set per layer application,
    smear gate from the context's first token, XSA, gate, lanes, adapters)."""
    cfg, w = _motif_cfg_weights()
    _check_reset(cfg, w, with_updates, tensor_cores)


@pytest.mark.parametrize("with_updates", [False, True])
def test_reset_logits_match_oracle(with_updates):
    cfg = ModelConfig(**SMALL)
    _check_reset(cfg, C.synth_weights(cfg, seed=21), with_updates, True)


def _check_reset(cfg, w, with_updates, tensor_cores):
    from altxs_b200 import _lib
    from altxs_b200.engine import ContextReset, DeviceModel, StreamBatch
    from altxs_b200.ttt import LoraTTT

    dm = DeviceModel(w, DEV, tensor_cores=tensor_cores)
    om = OracleModel(OracleWeights.from_model_weights(w))
    ottt = OracleTTT(om)
    rng = np.random.default_rng(5)
    T = 150  # segments [0,64), [64,128), [128,150)
    s = rng.integers(0, cfg.vocab_size, size=T)
    b = StreamBatch(dm, 1, words_per_stream=8, keep_logits=True, hist_len=cfg.ctx + 2)
    reset, ttt = ContextReset(dm), LoraTTT(dm)
    every = cfg.online_retrain_every
    st = om.new_stream()
    errs = []
    for t in range(T):
        if t > 0 and t % every == 0:
            idx = torch.arange(t - cfg.ctx - 1 if t > cfg.ctx else 0, t, device=DEV)
            b.hist[0, idx % b.hist_len] = torch.as_tensor(s[idx.cpu().numpy()], dtype=torch.int32, device=DEV)
            if with_updates:
                ttt(b, [0], t)
                ottt.update(s, t)
            reset(b, [0], t)
            st = om.reset_segment(s, t, ottt.lora if with_updates else None)
        tok = -1 if t == 0 else int(s[t - 1])
        b.tok.fill_(tok)
        if b.prev_tok is not None:  # LOGITS mode leaves the smear gate's previous token to the caller
            b.prev_tok.fill_(int(s[t - 2]) if t >= 2 else -1)
        b.step(_lib.STEP_LOGITS)
        got = b.logits[0].cpu().numpy()
        if tok >= 0:
            b.pos.add_(1)
            ref = om.step(st, tok, ottt.lora if with_updates else None).numpy()
            errs.append(float(np.abs(got - ref).max()))
    assert max(errs) < TOL, max(errs)
    assert int(b.pos.item()) == cfg.block_size - 1 + (T - 128)  # positions restarted at the last boundary


def test_reset_engine_roundtrip_with_motifs():
    from altxs_b200.engine import DeviceModel, Engine
    from altxs_b200.ttt import LoraTTT

    cfg, w = _motif_cfg_weights()
    dm = DeviceModel(w, DEV)
    rng = np.random.default_rng(8)
    streams = [rng.integers(0, cfg.vocab_size, size=k).astype(np.int32) for k in (200, 131)]
    enc = Engine(dm, ttt=LoraTTT(dm)).encode(streams)
    dec = Engine(dm, ttt=LoraTTT(dm)).decode([r.payload for r in enc], [len(x) for x in streams])
    for a, d in zip(streams, dec):
        assert np.array_equal(a, d)


@pytest.mark.parametrize("n_streams", [1, 3])
def test_reset_engine_roundtrip(n_streams):
    from altxs_b200.engine import DeviceModel, Engine
    from altxs_b200.synth import zipf_markov
    from altxs_b200.ttt import LoraTTT

    cfg = ModelConfig(**SMALL)
    dm = DeviceModel(C.synth_weights(cfg, seed=9), DEV)
    lens = [200, 131, 64][:n_streams]
    src = zipf_markov(max(lens), cfg.vocab_size, np.arange(n_streams) + 3)
    streams = [src[i, : lens[i]] for i in range(n_streams)]
    enc = Engine(dm, ttt=LoraTTT(dm)).encode(streams)
    dec = Engine(dm, ttt=LoraTTT(dm)).decode([r.payload for r in enc], lens)
    for a, d in zip(streams, dec):
        assert np.array_equal(a, d)
    # without updates too (context reset alone)
    enc2 = Engine(dm).encode(streams)
    dec2 = Engine(dm).decode([r.payload for r in enc2], lens)
    for a, d in zip(streams, dec2):
        assert np.array_equal(a, d)
