"""A decoder whose settings differ from the encoder's refuses the payload
(instead of desyncing silently), through the engine and the entry points."""

from __future__ import annotations

import struct

import numpy as np
import pytest
import torch

from altxs_b200 import codec as C
from altxs_b200 import lockstep
from altxs_b200.config import ModelConfig

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
SMALL = dict(vocab_size=512, num_layers=2, model_dim=128, num_heads=4, num_kv_heads=2, block_size=32,
             online_retrain_every=64, seed=11, ttt_lora_rank=4, ttt_k_lora=True, ttt_o_lora=True)


def _streams(cfg, n=2, length=150):
    rng = np.random.default_rng(3)
    return [rng.integers(0, cfg.vocab_size, size=length).astype(np.int32) for _ in range(n)]


def test_decoder_on_the_other_linear_path_is_refused():
    from altxs_b200.engine import DeviceModel, Engine
    from altxs_b200.ttt import LoraTTT

    cfg = ModelConfig(**SMALL)
    w = C.synth_weights(cfg, seed=2)
    tc, cc = DeviceModel(w, DEV, tensor_cores=True), DeviceModel(w, DEV, tensor_cores=False)
    streams = _streams(cfg)
    enc = Engine(tc, ttt=LoraTTT(tc)).encode(streams)
    with pytest.raises(lockstep.LockstepMismatch, match="linear_path"):
        Engine(cc, ttt=LoraTTT(cc)).decode([r.payload for r in enc], [len(s) for s in streams])
    # without the update on the decoder side
    with pytest.raises(lockstep.LockstepMismatch, match="online_retrain_enabled"):
        Engine(tc).decode([r.payload for r in enc], [len(s) for s in streams])
    # the matching decoder round-trips
    dec = Engine(tc, ttt=LoraTTT(tc)).decode([r.payload for r in enc], [len(s) for s in streams])
    for s, d in zip(streams, dec):
        assert np.array_equal(s, d)


def test_payload_without_header_still_decodes():
    from altxs_b200.engine import DeviceModel, Engine

    cfg = ModelConfig(**{**SMALL, "retrain_mode": "none"})
    dm = DeviceModel(C.synth_weights(cfg, seed=2), DEV)
    streams = _streams(cfg)
    enc = Engine(dm).encode(streams)
    bare = []
    for r in enc:
        _, fp, body = lockstep.split_header(r.payload)
        assert fp is not None
        bare.append(body)
    assert bare[0] == b"".join(struct.pack("<Q", len(p)) + p for p in enc[0].segments)
    dec = Engine(dm).decode(bare, [len(s) for s in streams])
    for s, d in zip(streams, dec):
        assert np.array_equal(s, d)


def test_entry_points_refuse_another_cdf_rule_or_other_weights():
    from altxs_b200.incremental import compress_full_sha_incremental, decompress_full_sha_incremental

    cfg = ModelConfig(**SMALL)
    w = C.synth_weights(cfg, seed=2)
    data = _streams(cfg, 1, 200)[0]
    res = compress_full_sha_incremental(w, data, cfg=cfg, device=DEV, progress=False)
    other = ModelConfig(**{**SMALL, "cdf_mode": "ref"})
    with pytest.raises(lockstep.LockstepMismatch, match="cdf_mode"):
        decompress_full_sha_incremental(C.synth_weights(other, seed=2), res["payload"], len(data), cfg=other,
                                        device=DEV, progress=False)
    with pytest.raises(lockstep.LockstepMismatch, match="weights_sha256"):
        decompress_full_sha_incremental(C.synth_weights(cfg, seed=3), res["payload"], len(data), cfg=cfg,
                                        device=DEV, progress=False)
    ok = decompress_full_sha_incremental(w, res["payload"], len(data), cfg=cfg, device=DEV, progress=False)
    assert ok["decoded_sha256"] == res["sha256"]
