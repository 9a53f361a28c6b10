"""The fused step (one persistent cooperative kernel per symbol step for a few
streams on the CUDA-core path; off by default) against the launch-per-phase
step: identical logits and identical bitstreams, plain and motif models, with
adapters; one launch per step; its bounded grid barrier gives up cleanly."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from altxs_b200 import _lib
from altxs_b200 import codec as C
from altxs_b200.config import ModelConfig

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")

SMALL = dict(
    vocab_size=512, num_layers=3, model_dim=128, num_heads=4, num_kv_heads=2, mlp_mult=4.0, rope_dims=16,
    block_size=32, online_retrain_every=64, seed=11, ttt_lora_rank=4, ttt_lora_lr=1e-3, ttt_k_lora=True,
    ttt_o_lora=True,
)
# head_dim 64, one query head per KV head (the benchmark model's head shape), small vocab
WIDE = dict(
    vocab_size=1024, num_layers=2, model_dim=512, num_heads=8, num_kv_heads=8, mlp_mult=4.0, rope_dims=16,
    block_size=48, online_retrain_every=64, seed=3, ttt_lora_rank=8, ttt_lora_lr=1e-3, ttt_k_lora=True,
    ttt_o_lora=True,
)


def _model(name):
    from altxs_b200.engine import DeviceModel

    if name == "plain":
        cfg = ModelConfig(**SMALL)
        w = C.synth_weights(cfg, seed=6)
    elif name == "wide":
        cfg = ModelConfig(**WIDE)
        w = C.synth_weights(cfg, seed=6)
    elif name == "mlp_lora":
        cfg = ModelConfig(**{**SMALL, "ttt_lora_rank": 80, "ttt_k_lora": False, "ttt_mlp_lora": True,
                             "ttt_o_lora_on_y": True})
        w = C.synth_weights(cfg, seed=6)
    else:  # every motif, adapters on every slot
        from tests.test_gpu_lora_motifs import _cfg, _weights

        cfg = _cfg("all")
        w = _weights(cfg, seed=6)
    return cfg, DeviceModel(w, DEV, tensor_cores=False)


def _encode(dm, streams, fused: bool, ttt: bool):
    from altxs_b200.engine import Engine
    from altxs_b200.ttt import LoraTTT

    L = _lib.lib()
    assert L.altxs_set_step_fusion(4 if fused else 0) == 0
    try:
        return Engine(dm, ttt=LoraTTT(dm) if ttt else None).encode(streams)
    finally:
        L.altxs_set_step_fusion(0)


@pytest.mark.parametrize("n", [1, 2, 4])
@pytest.mark.parametrize("name", ["plain", "wide", "mlp_lora", "motifs"])
def test_fused_step_bitstreams_identical(name, n):
    """Encode with LoRA updates at the boundaries: the fused step's bitstreams
    equal the launch-per-phase step's, byte for byte; decode round-trips."""
    from altxs_b200.engine import Engine
    from altxs_b200.ttt import LoraTTT

    cfg, dm = _model(name)
    rng = np.random.default_rng(n)
    streams = [rng.integers(0, cfg.vocab_size, size=int(k)).astype(np.int32)
               for k in rng.integers(70, 150, size=n)]
    a = _encode(dm, streams, fused=True, ttt=True)
    b = _encode(dm, streams, fused=False, ttt=True)
    for x, y in zip(a, b):
        assert x.payload == y.payload
    back = Engine(dm, ttt=LoraTTT(dm)).decode([r.payload for r in a], [len(s) for s in streams])
    for s, d in zip(streams, back):
        assert np.array_equal(s, d)


@pytest.mark.parametrize("name", ["plain", "wide", "motifs"])
def test_fused_step_logits_identical_and_one_launch(name):
    """LOGITS mode over the window with random adapters: the fused step's logits
    equal the launch-per-phase step's bit for bit, and a step is one launch."""
    from altxs_b200.engine import StreamBatch
    from tests.test_gpu_step import _lora_vec

    cfg, dm = _model(name)
    L = _lib.lib()
    vec, _ = _lora_vec(cfg, np.random.default_rng(3))
    toks = np.random.default_rng(4).integers(0, cfg.vocab_size, size=(2, cfg.block_size + 6))
    outs = []
    for fused in (True, False):
        assert L.altxs_set_step_fusion(4 if fused else 0) == 0
        try:
            b = StreamBatch(dm, 2, words_per_stream=8, keep_logits=True)
            b.lora.copy_(torch.as_tensor(vec, device=DEV).expand_as(b.lora))
            got = []
            for t in range(toks.shape[1]):
                b.tok.copy_(torch.as_tensor(toks[:, t], dtype=torch.int32, device=DEV))
                if b.prev_tok is not None:
                    b.prev_tok.copy_(torch.as_tensor(toks[:, t - 1] if t else [-1, -1], dtype=torch.int32,
                                                     device=DEV))
                torch.cuda.synchronize()
                n0 = int(L.altxs_launch_count())
                b.step(_lib.STEP_LOGITS)
                launches = int(L.altxs_launch_count()) - n0
                if fused:
                    assert launches == 1, launches
                else:
                    assert launches > 10, launches
                got.append(b.logits.cpu().numpy().copy())
                b.pos.add_(1)
            outs.append(np.stack(got))
        finally:
            L.altxs_set_step_fusion(0)
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


def test_fused_step_timeout_reports_and_recovers():
    """With the TMA wait limit at 0 the fused step's attention gives up: every
    stream is marked ALTXS_ST_TIMEOUT, all blocks leave through the bounded grid
    barrier, and the next steps run normally."""
    from altxs_b200.engine import Engine, StreamBatch

    cfg, dm = _model("plain")
    L = _lib.lib()
    assert L.altxs_set_step_fusion(4) == 0
    try:
        b = StreamBatch(dm, 2, words_per_stream=64)
        b.ac_init()
        syms = np.random.default_rng(0).integers(0, cfg.vocab_size, size=(2, 8))
        for t in range(4):
            b.sym.copy_(torch.as_tensor(syms[:, t], dtype=torch.int32, device=DEV))
            b.step(_lib.STEP_ENCODE)
        torch.cuda.synchronize()
        assert all(s == 0 for s in b.status())
        try:
            assert L.altxs_set_wait_limit(0) == 0
            b.sym.copy_(torch.as_tensor(syms[:, 4], dtype=torch.int32, device=DEV))
            b.step(_lib.STEP_ENCODE)
            torch.cuda.synchronize()
        finally:
            assert L.altxs_set_wait_limit(L.altxs_default_wait_limit()) == 0
        assert all(s & _lib.ST_TIMEOUT for s in b.status())
        streams = [syms[0], syms[1, :5]]
        enc = Engine(dm).encode(streams)
        dec = Engine(dm).decode([r.payload for r in enc], [len(x) for x in streams])
        for a, d in zip(streams, dec):
            assert np.array_equal(a, d)
    finally:
        L.altxs_set_step_fusion(0)
