"""Host-side pins of config C1: the synthetic stream and the seed-0 weights
are the ones the reference fixtures were made from."""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

from altxs_b200 import codec as C
from altxs_b200.config import c1_config
from altxs_b200.synth import zipf_markov

GOLD = Path(__file__).resolve().parent / "golden"
BANKS = ("tok_emb.weight", "qo_bank", "kv_bank", "mlp_up_bank", "mlp_down_bank")


def test_c1_stream_is_the_fixture_stream():
    g = np.load(GOLD / "c1_stream.npz")
    arr = zipf_markov(65536, 4096, [1])[0]
    assert hashlib.sha256(arr.astype("<u2").tobytes()).digest() == g["stream_sha"].tobytes()


def test_c1_weights_are_the_reference_seed0_init():
    """``reference_init`` replays the reference GPT's construction draws; its
    banks hash to those of ``torch.manual_seed(0); GPT(cfg)``."""
    g = np.load(GOLD / "c1_stream.npz")
    w = C.reference_init(c1_config(), 0)
    h = hashlib.sha256()
    for k in BANKS:
        h.update(np.ascontiguousarray(w[k], dtype=np.float32).tobytes())
    assert h.digest() == g["bank_sha"].tobytes()


def test_reference_fixtures_are_consistent():
    g = np.load(GOLD / "c1_stream.npz")
    i = np.load(GOLD / "incr_stream.npz")
    assert np.array_equal(g["row_pos"], i["row_pos"])
    assert int(g["retrain_count"]) == 15 and int(i["replenish_retrain_count"]) == 15
    # bits/symbol is payload bytes * 8 / n in the reference's result dicts
    for bits, nbytes in ((g["bits_per_symbol"], g["payload_bytes"]),
                         (i["none_bits_per_symbol"], i["none_payload_bytes"]),
                         (i["replenish_bits_per_symbol"], i["replenish_payload_bytes"])):
        assert abs(float(bits) - int(nbytes) * 8 / 65536) < 1e-12
    # rows are normalised log-probabilities
    for rows in (g["row_logp"], i["none_row_logp"], i["replenish_row_logp"]):
        assert np.allclose(np.exp(rows.astype(np.float64)).sum(axis=1), 1.0, atol=1e-4)
