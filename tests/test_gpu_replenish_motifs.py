"""Full-parameter retraining of a model with the reference motifs on (smear
gate, XSA, sparse attention gate, asymmetric softcap, depth loops, parallel
lanes) on the B200 kernels: every parameter's gradient against torch
autograd on the oracle, both retrain modes against the reference's own
online_retrain (golden), and encode -> decode lockstep through the engine."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from altxs_b200 import _lib
from altxs_b200 import codec as C
from altxs_b200.config import ModelConfig
from oracle.replenish import OracleReplenish
from tests.test_gpu_motifs import BASE, CASES
from tests.test_gpu_replenish import _model, _rel_err
from tests.test_oracle_golden import motif_case

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _motif_model(name: str, tensor_cores: bool):
    """Synthetic mixed-bit weights with random motif parameters, in a parameter arena."""
    from altxs_b200.engine import DeviceModel

    kw = dict(BASE)
    kw.update(CASES[name])
    kw["retrain_mode"] = "replenish"
    cfg = ModelConfig(**kw)
    w = C.synth_weights(cfg, seed=9)
    rng = np.random.default_rng(len(name))
    s = w.small
    s["smear_gate"] = rng.normal(0, 0.5, s["smear_gate"].shape).astype(np.float32)
    s["smear_lambda"] = np.array([0.7], dtype=np.float32)
    s["attn_gate_w"] = rng.normal(0, 0.5, s["attn_gate_w"].shape).astype(np.float32)
    s["softcap"] = np.array([12.0, 20.0], dtype=np.float32)
    s["parallel_post"] = (s["parallel_post"] + rng.normal(0, 0.1, s["parallel_post"].shape)).astype(np.float32)
    s["parallel_resid"] = (s["parallel_resid"] + rng.normal(0, 0.1, s["parallel_resid"].shape)).astype(np.float32)
    s["skip_gates"] = (s["skip_gates"] + rng.normal(0, 0.3, s["skip_gates"].shape)).astype(np.float32)
    return cfg, DeviceModel(w, DEV, tensor_cores=tensor_cores, full_params=True)


def _loss_grad(dm, ids, first):
    L = _lib.lib()
    n = len(ids)
    dm.ensure_rope(n + 1)
    wsb = L.altxs_full_workspace_bytes(ctypes.byref(dm.desc), n)
    assert wsb > 0
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
    grad = torch.full((dm.layout.total,), float("nan"), device=DEV)
    loss = torch.zeros(1, device=DEV)
    tok = torch.as_tensor(ids, device=DEV)
    rc = L.altxs_full_loss_grad(ctypes.byref(dm.desc), ctypes.byref(dm.weights_struct),
                                ctypes.byref(dm.dense_weights()), tok.data_ptr(), n, first, loss.data_ptr(),
                                grad.data_ptr(), ws.data_ptr(), wsb, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    return float(loss), grad


@pytest.mark.parametrize("tensor_cores", [False, True])
@pytest.mark.parametrize("name", list(CASES))
def test_motif_gradient_matches_autograd(name, tensor_cores):
    """Loss and d(loss)/d(every parameter), the motifs' own included, of one
    window (unscored context rows before `first`) against torch autograd on
    the oracle forward of the same weights.  Depth loops add a layer's
    applications; parallel lanes split and rejoin the stream."""
    from altxs_b200.replenish import state_from_arena

    cfg, dm = _motif_model(name, tensor_cores)
    ids = np.random.default_rng(3).integers(0, cfg.vocab_size, size=41).astype(np.int32)
    first = 9
    loss, grad = _loss_grad(dm, ids, first)
    assert torch.isfinite(grad).all()  # every entry written
    st = state_from_arena(dm)
    o = OracleReplenish(cfg, st)
    ref_loss = o.window_ce(ids, first)
    ref_loss.backward()
    ref = {k: p.grad.numpy() for k, p in o.p.items()}
    got = state_from_arena(dm, grad)
    assert set(ref) <= set(got)
    assert abs(loss - float(ref_loss.detach())) < (1e-5 if not tensor_cores else 2e-4)
    err = _rel_err(got, ref)
    assert err < (2e-4 if not tensor_cores else 3e-3), err


@pytest.mark.parametrize("tensor_cores", [False, True])
@pytest.mark.parametrize("case", ["m_full", "m_xm"])
def test_motif_retrain_matches_reference(golden, case, tensor_cores):
    """The reference's "full" mode (replay windows) and replenish (Forward-XM)
    on its motif model, four boundaries through the device kernels: the loss of
    every boundary, the XM choice, and the final weights in units of an
    optimizer step (Adam turns a near-zero gradient's sign into a full step)."""
    from altxs_b200.replenish import ReplenishTTT, state_from_arena

    g = golden("motif_retrain.npz")
    cfg, w0 = motif_case(g, case)
    dm = _model(cfg, w0, tensor_cores)
    ttt = ReplenishTTT(dm, n_total=len(g["arr"]))
    prefix = torch.as_tensor(g["arr"].astype(np.int32), device=DEV)
    diffs = []
    for end in (24, 48, 72, 96):
        ttt.boundary(prefix, end)
        diffs.append(abs(float(ttt.loss[0]) - float(g[f"{case}/{end}/loss"])))
        if f"{case}/{end}/xm_chosen" in g.files:
            assert ttt.xm_last["chosen"] == int(g[f"{case}/{end}/xm_chosen"]), (end, ttt.xm_last["scores"])
            assert np.abs(np.array(ttt.xm_last["scores"]) - g[f"{case}/{end}/xm_scores"]).max() < 1e-3
    torch.cuda.synchronize()
    print(case, "tc" if tensor_cores else "fp32", "loss diffs", diffs)
    # the first boundary pins the model; later ones carry the earlier steps' drift
    # (two AdamW steps per boundary with beta1 0.9 in m_full)
    assert diffs[0] < (2e-4 if tensor_cores else 2e-5), diffs
    assert max(diffs) < (5e-4 if tensor_cores else 1e-4), diffs
    got = state_from_arena(dm)
    ref = {k[len(case) + 3:]: g[k] for k in g.files if k.startswith(f"{case}/w/")}
    assert set(ref) <= set(got)
    lr = float(cfg.ttt_lora_lr)
    worst = max(float(np.abs(got[k] - v).max()) for k, v in ref.items())
    assert worst < (1.5 if tensor_cores else 0.5) * lr, (worst, lr)


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_motif_replenish_round_trip(tensor_cores):
    """Encode -> decode through the engine with every motif on and a
    full-parameter update (Forward-XM) at each boundary: bit-exact round trip,
    encoder and decoder models bit-identical afterwards."""
    from altxs_b200.engine import DeviceModel, Engine
    from altxs_b200.replenish import ReplenishTTT

    kw = dict(BASE)
    kw.update(CASES["all"])
    kw.update(retrain_mode="replenish", block_size=24, online_retrain_every=40, ttt_lora_lr=3e-3,
              ttt_replenish_warmup_steps=1, ttt_replenish_xm_4x_until_bytes=100)
    cfg = ModelConfig(**kw)
    w = C.synth_weights(cfg, seed=4)
    rng = np.random.default_rng(3)
    # each stream crosses >= 2 boundaries: the first is a warmup one (lr 0, the model stays)
    streams = [rng.integers(0, cfg.vocab_size, size=k).astype(np.int32) for k in (130, 97)]
    enc_dm = DeviceModel(w, DEV, tensor_cores=tensor_cores, full_params=True)
    enc = Engine(enc_dm, ttt=ReplenishTTT(enc_dm))
    res = enc.encode(streams)
    p_enc = enc_dm.params.clone()
    dec_dm = DeviceModel(w, DEV, tensor_cores=tensor_cores, full_params=True)
    dec = Engine(dec_dm, ttt=ReplenishTTT(dec_dm))
    back = dec.decode([r.payload for r in res], [len(s) for s in streams])
    for s, d in zip(streams, back):
        assert np.array_equal(s, d)
    assert torch.equal(p_enc, dec_dm.params)
    assert not torch.equal(p_enc, enc.ttt.initial)
