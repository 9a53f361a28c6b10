"""The allocation-free step entry point agrees with the regular one.

``altxs_step_noalloc`` serves callers that cannot allocate device memory (a
host framework that owns the device budget, or a caller that must not risk an
allocation's device-wide synchronisation): it takes no workspace and uses a
fixed scratch array inside the library instead.  This file runs last (its
name sorts after the others) and also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from altxs_b200 import codec as C_
from altxs_b200.config import ModelConfig

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")

SMALL = dict(
    vocab_size=512, num_layers=3, model_dim=128, num_heads=4, num_kv_heads=2,
    mlp_mult=4.0, rope_dims=16, block_size=32, online_retrain_every=64, seed=11,
    ttt_lora_rank=4, ttt_k_lora=True, ttt_o_lora=True,
)


def _call(L, fn, dm, b, mode):
    return fn(C.byref(dm.desc), C.byref(dm.weights_struct), C.byref(b._batch), mode,
              torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("tensor_cores,fusion,n", [(True, 0, 6), (False, 0, 6), (False, 4, 3)])
def test_noalloc_step_matches_regular_step_two_calls(tensor_cores, fusion, n):
    """Both linear paths, and the fused persistent step (whose grid-barrier
    words live in the same scratch), give bit-identical logits, coder states
    and bitstreams through either entry point: the kernels are the same and
    only the scratch address differs."""
    from altxs_b200 import _lib
    from altxs_b200.engine import DeviceModel, StreamBatch
    from altxs_b200.synth import zipf_markov

    L = _lib.lib()
    cfg = ModelConfig(**SMALL)
    dm = DeviceModel(C_.synth_weights(cfg, seed=4), DEV, tensor_cores=tensor_cores)
    T = 40
    syms = zipf_markov(T, cfg.vocab_size, np.arange(n) + 3)
    a = StreamBatch(dm, n, words_per_stream=64, keep_logits=True)
    b = StreamBatch(dm, n, words_per_stream=64, keep_logits=True)
    assert L.altxs_set_step_fusion(fusion) == 0
    try:
        # bring both batches to the same mid-stream state with the regular step
        for t in range(T - 2):
            a.sym.copy_(torch.as_tensor(syms[:, t], device=DEV))
            a.step(_lib.STEP_ENCODE)
        for name in ("tok", "pos", "kv", "ac", "bits", "lora"):
            getattr(b, name).copy_(getattr(a, name))
        # two calls in a row: regular entry point on a, allocation-free one on b
        for t in (T - 2, T - 1):
            s = torch.as_tensor(syms[:, t], device=DEV)
            a.sym.copy_(s)
            b.sym.copy_(s)
            assert _call(L, L.altxs_step, dm, a, _lib.STEP_ENCODE) == 0
            assert _call(L, L.altxs_step_noalloc, dm, b, _lib.STEP_ENCODE) == 0
            torch.cuda.synchronize()
            assert torch.isfinite(b.logits).all()
            assert torch.equal(a.logits.view(torch.int32), b.logits.view(torch.int32))
            assert torch.equal(a.ac, b.ac)  # coder states (integer) identical
            assert torch.equal(a.pos, b.pos) and torch.equal(a.tok, b.tok)
    finally:
        L.altxs_set_step_fusion(0)
    a.ac_flush()
    b.ac_flush()
    assert a.segment_bytes(list(range(n))) == b.segment_bytes(list(range(n)))
    a.check_status()
    b.check_status()


def test_noalloc_step_rejects_batches_beyond_its_scratch():
    from altxs_b200 import _lib
    from altxs_b200.config import c3_config
    from altxs_b200.engine import DeviceModel

    L = _lib.lib()
    cap = L.altxs_step_noalloc_max_bytes()
    assert cap == 16 << 20
    dm = DeviceModel(C_.synth_weights(c3_config(), seed=1), DEV)
    n = 1
    while L.altxs_workspace_bytes(C.byref(dm.desc), n) <= cap:
        n *= 2
    batch = _lib.Batch(n_streams=n)  # the size check happens before any pointer is used
    rc = L.altxs_step_noalloc(C.byref(dm.desc), C.byref(dm.weights_struct), C.byref(batch), _lib.STEP_LOGITS,
                              torch.cuda.current_stream().cuda_stream)
    assert rc == -28  # ALTXS_ENOSPC
