"""Bounded device waits: with the first-wait limit at 0 every pipeline wait
of a real step gives up; the kernels record ALTXS_ST_TIMEOUT in the streams'
status words, drain their own copies and MMAs, free tensor memory and return.
No fault, no hang, and the context keeps working afterwards."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from altxs_b200 import codec as C
from altxs_b200.config import ModelConfig

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")

SMALL = dict(
    vocab_size=512, num_layers=3, model_dim=128, num_heads=4, num_kv_heads=2,
    mlp_mult=4.0, rope_dims=16, block_size=32, online_retrain_every=64, seed=11,
    ttt_lora_rank=4, ttt_k_lora=True, ttt_o_lora=True,
)


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_waits_give_up_report_and_recover(tensor_cores):
    from altxs_b200 import _lib
    from altxs_b200.engine import DeviceModel, Engine, StreamBatch
    from altxs_b200.synth import zipf_markov

    L = _lib.lib()
    cfg = ModelConfig(**SMALL)
    dm = DeviceModel(C.synth_weights(cfg, seed=6), DEV, tensor_cores=tensor_cores)
    n = 3
    syms = zipf_markov(12, cfg.vocab_size, np.arange(n) + 2)
    b = StreamBatch(dm, n, words_per_stream=64)
    b.ac_init()
    for t in range(6):
        b.sym.copy_(torch.as_tensor(syms[:, t], device=DEV))
        b.step(_lib.STEP_ENCODE)
    torch.cuda.synchronize()
    assert all(s == 0 for s in b.status())
    try:
        assert L.altxs_set_wait_limit(0) == 0
        b.sym.copy_(torch.as_tensor(syms[:, 6], device=DEV))
        b.step(_lib.STEP_ENCODE)
        torch.cuda.synchronize()
    finally:
        assert L.altxs_set_wait_limit(L.altxs_default_wait_limit()) == 0
    st = b.status()
    assert all(s & _lib.ST_TIMEOUT for s in st), st
    with pytest.raises(RuntimeError):
        b.check_status()
    # same process, same device: a fresh encode/decode round trip is unaffected
    lens = [40, 25]
    src = zipf_markov(40, cfg.vocab_size, np.array([5, 9]))
    streams = [src[i, : lens[i]] for i in range(2)]
    enc = Engine(dm).encode(streams)
    dec = Engine(dm).decode([r.payload for r in enc], lens)
    for a, d in zip(streams, dec):
        assert np.array_equal(a, d)
