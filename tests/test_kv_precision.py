"""KV-cache storage precision at the 33M shapes with the window full.

The decode step keeps each K/V value as 24 bits (fp32 rounded to nearest
even at bit 8: a bf16 high part plus the next 8 mantissa bits).  This test
measures, on the CPU oracle, what each storage format does to the logits when
every one of the 2048 window rows is read: a stream of 2100 symbols (the ring
wraps, every 256-key split is full), positions 2040..2099 compared with the
unrounded fp32 oracle.  fp16 and bf16 rows move the logits past the 2e-3
parity bar; the 24-bit rows stay well inside it.
"""

from __future__ import annotations

import numpy as np
import torch

from altxs_b200 import codec as C
from altxs_b200.config import c3_config
from altxs_b200.synth import zipf_markov
from oracle.model import OracleModel, OracleWeights

T, FIRST = 2100, 2040


def round24(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> 24 bits (sign, exponent, 15 mantissa bits), round to nearest even."""
    b = x.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    b = (b + 0x7F + ((b >> 8) & 1)) & 0xFFFFFF00
    b = torch.where(b >= 1 << 31, b - (1 << 32), b)
    return b.to(torch.int32).view(torch.float32)


def _logits(om, toks):
    st = om.new_stream()
    out = [om.prefill(st, toks[:FIRST]).numpy()]
    for t in range(FIRST, T - 1):
        out.append(om.step(st, int(toks[t])).numpy())
    return np.stack(out)


def test_kv_storage_formats_at_full_window():
    cfg = c3_config()
    om = OracleModel(OracleWeights.from_model_weights(C.synth_weights(cfg, seed=1)))
    toks = zipf_markov(T, cfg.vocab_size, [5])[0]
    exact = _logits(om, toks)
    err = {}
    for name, fn in (("24-bit", round24),
                     ("fp16", lambda x: x.half().float()),
                     ("bf16", lambda x: x.bfloat16().float())):
        om.kv_round = fn
        err[name] = float(np.abs(_logits(om, toks) - exact).max())
    om.kv_round = None
    print("max |logit error| by KV format:", err)
    assert err["24-bit"] < 1e-3
    assert err["fp16"] > 2e-3 and err["bf16"] > 2e-3


def test_round24_is_round_to_nearest_even():
    x = torch.tensor([1.0, 1.0 + 2.0 ** -16, 1.0 + 3 * 2.0 ** -16, -2.5, 3.0e-30, 1.0 + 2.0 ** -15 + 2.0 ** -23],
                     dtype=torch.float32)
    y = round24(x)
    assert y[0] == 1.0 and y[3] == -2.5
    assert y[1] == 1.0  # tie, mantissa even: down
    assert y[2] == 1.0 + 4 * 2.0 ** -16  # tie, odd: up
    assert y[5] == 1.0 + 2.0 ** -15  # below the halfway point: down
    b = y.view(torch.int32)
    assert bool(((b & 0xFF) == 0).all())
