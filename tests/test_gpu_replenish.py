"""Full-parameter replenish on the B200 kernels: the gradient of every
parameter against torch autograd on the oracle, whole boundaries (Forward-XM,
anchor, anneal, replay) against the reference's own online_retrain (golden),
and encode -> decode lockstep through the engine."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from altxs_b200 import _lib
from altxs_b200 import codec as C
from oracle.replenish import OracleReplenish
from tests.test_oracle_golden import replenish_case

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
CASES = ["xm", "xm_probe2_anchor", "replay"]


def _model(cfg, state, tensor_cores):
    from altxs_b200.engine import DeviceModel

    w = C.dense_weights(cfg, {k: np.asarray(v, dtype=np.float32) for k, v in state.items()})
    return DeviceModel(w, DEV, tensor_cores=tensor_cores, full_params=True)


def _rel_err(got: dict, ref: dict) -> float:
    """Largest |got - ref| over every tensor, relative to that tensor's largest |ref|."""
    worst = 0.0
    for k, r in ref.items():
        scale = max(float(np.abs(r).max()), 1e-12)
        worst = max(worst, float(np.abs(got[k] - r).max()) / scale)
    return worst


@pytest.mark.parametrize("tensor_cores", [False, True])
@pytest.mark.parametrize("n,first", [(40, 15), (33, 0), (17, 5)])
def test_full_gradient_matches_autograd(golden, tensor_cores, n, first):
    """Loss and d(loss)/d(every parameter) of one chunk window (context rows
    before `first` unscored; odd window lengths) against torch autograd on the
    oracle forward.  CUDA cores: fp32 arithmetic; tensor cores: hi/lo bf16
    products (2^-16 relative), so the bound is looser."""
    from altxs_b200.replenish import state_from_arena

    g = golden("replenish.npz")
    cfg, w0, _ = replenish_case(g, "xm")
    dm = _model(cfg, w0, tensor_cores)
    L = _lib.lib()
    rng = np.random.default_rng(n)
    ids = rng.integers(0, cfg.vocab_size, size=n).astype(np.int32)
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
    assert torch.isfinite(grad).all()  # every entry written

    o = OracleReplenish(cfg, w0)
    ref_loss = o.window_ce(ids, first)
    ref_loss.backward()
    ref = {k: p.grad.numpy() for k, p in o.p.items()}
    got = state_from_arena(dm, grad)
    assert abs(float(loss) - float(ref_loss.detach())) < (1e-5 if not tensor_cores else 2e-4)
    err = _rel_err(got, ref)
    assert err < (1e-4 if not tensor_cores else 3e-3), err


@pytest.mark.parametrize("tensor_cores", [False, True])
@pytest.mark.parametrize("case", CASES)
def test_replenish_boundaries_match_reference(golden, case, tensor_cores):
    """Four boundaries of the reference's online_retrain in replenish mode,
    run through the device kernels: the XM choice at every boundary equals the
    reference's, the probe scores agree, and the final weights agree."""
    from altxs_b200.replenish import ReplenishTTT, state_from_arena

    g = golden("replenish.npz")
    cfg, w0, masks = replenish_case(g, case)
    dm = _model(cfg, w0, tensor_cores)
    arr = g["arr"]
    ttt = ReplenishTTT(dm, n_total=len(arr), anchor_masks=masks)
    prefix = torch.as_tensor(arr.astype(np.int32), device=DEV)
    for end in (24, 48, 72, 96):
        ttt.boundary(prefix, end)
        torch.cuda.synchronize()
        key = f"{case}/{end}/xm_chosen"
        if key in g.files:
            assert ttt.xm_last["end"] == end
            assert ttt.xm_last["chosen"] == int(g[key]), (end, ttt.xm_last["scores"], g[f"{case}/{end}/xm_scores"])
            assert np.abs(np.array(ttt.xm_last["scores"]) - g[f"{case}/{end}/xm_scores"]).max() < 1e-3
    got = state_from_arena(dm)
    ref = {k[len(case) + 3:]: g[k] for k in g.files if k.startswith(f"{case}/w/")}
    ref = {k: v for k, v in ref.items() if k in got}
    lr = float(cfg.ttt_lora_lr)
    worst = max(float(np.abs(got[k] - v).max()) for k, v in ref.items())
    # Adam moves every weight by about lr per step, so a disagreement is measured
    # in steps: fp32 agrees to a few percent of one step; the tensor cores' 2^-16
    # products reach a near-zero gradient's sign, within half a step here
    assert worst < (0.5 if tensor_cores else 0.05) * lr, (worst, lr)


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_replenish_engine_round_trip(tensor_cores):
    """Encode -> decode through the engine with a full-parameter update at
    every boundary (Forward-XM on): bit-exact round trip, and the decoder's
    model ends bit-identical to the encoder's (lockstep)."""
    from altxs_b200.config import ModelConfig
    from altxs_b200.engine import DeviceModel, Engine
    from altxs_b200.replenish import ReplenishTTT

    cfg = ModelConfig(vocab_size=96, num_layers=2, model_dim=64, num_heads=4, num_kv_heads=2, mlp_mult=2.0,
                      rope_dims=8, block_size=24, online_retrain_every=40, retrain_mode="replenish",
                      ttt_lora_lr=3e-3, ttt_replenish_warmup_steps=1, ttt_replenish_xm_4x_until_bytes=100)
    w = C.synth_weights(cfg, seed=4)
    rng = np.random.default_rng(3)
    streams = [rng.integers(0, cfg.vocab_size, size=k).astype(np.int32) for k in (170, 81)]
    enc_dm = DeviceModel(w, DEV, tensor_cores=tensor_cores, full_params=True)
    enc = Engine(enc_dm, ttt=ReplenishTTT(enc_dm))
    res = enc.encode(streams)
    p_enc = enc_dm.params.clone()  # after the last stream
    dec_dm = DeviceModel(w, DEV, tensor_cores=tensor_cores, full_params=True)
    dec = Engine(dec_dm, ttt=ReplenishTTT(dec_dm))
    back = dec.decode([r.payload for r in res], [len(s) for s in streams])
    for s, d in zip(streams, back):
        assert np.array_equal(s, d)
    assert torch.equal(p_enc, dec_dm.params)
    assert enc.ttt.boundaries >= 5 and enc.ttt.xm_counts
    assert not torch.equal(p_enc, enc.ttt.initial)  # the updates did change the model


@pytest.mark.parametrize("tensor_cores", [False, True])
@pytest.mark.parametrize("case", ["full_plain", "full_replay", "full_burst"])
def test_full_retrain_matches_reference(golden, case, tensor_cores):
    """The reference's default "full" retrain mode through the device kernels
    (window loss of the last block, replay windows, burst steps on their own
    AdamW) against the reference's online_retrain: the loss of every
    boundary's last step, and the final weights in units of an optimizer step.
    A burst's first AdamW step (beta1 0.9, bias-corrected) moves every weight
    by about +-lr whatever its gradient's size, and it replays windows the
    model has already trained on, where many gradients are ~0 and their signs
    follow summation order; the losses pin the model itself."""
    from altxs_b200.replenish import ReplenishTTT, state_from_arena
    from tests.test_oracle_golden import full_case

    g = golden("full_retrain.npz")
    cfg, w0 = full_case(g, case)
    dm = _model(cfg, w0, tensor_cores)
    ttt = ReplenishTTT(dm, n_total=len(g["arr"]))
    prefix = torch.as_tensor(g["arr"].astype(np.int32), device=DEV)
    for end in (24, 48, 72, 96):
        ttt.boundary(prefix, end)
        loss = float(ttt.loss[0])
        assert abs(loss - float(g[f"{case}/{end}/loss"])) < (2e-4 if tensor_cores else 2e-5), (end, loss)
    torch.cuda.synchronize()
    got = state_from_arena(dm)
    ref = {k[len(case) + 3:]: g[k] for k in g.files if k.startswith(f"{case}/w/")}
    ref = {k: v for k, v in ref.items() if k in got}
    lr = max(cfg.ttt_lora_lr, cfg.ttt_burst_lr if cfg.ttt_burst_schedule else 0.0)
    worst = max(float(np.abs(got[k] - v).max()) for k, v in ref.items())
    assert worst < (1.5 if tensor_cores else 0.5) * lr, (worst, lr)


@pytest.mark.parametrize("mode", ["full", "replenish"])
def test_entry_points_with_full_parameter_update(mode):
    """The reference-mirroring entry points in the reference's default "full"
    mode and in replenish mode: the update trains every weight of the model at
    each boundary on both sides; verify_decode restores the input and a
    separate decompress call does too (both start from the shipped weights)."""
    from altxs_b200.config import ModelConfig
    from altxs_b200.incremental import compress_full_sha_incremental, decompress_full_sha_incremental

    cfg = ModelConfig(vocab_size=64, num_layers=2, model_dim=64, num_heads=4, num_kv_heads=2, mlp_mult=2.0,
                      rope_dims=8, block_size=16, online_retrain_every=40, retrain_mode=mode, ttt_lora_lr=2e-3,
                      online_retrain_steps=2, ttt_replenish_warmup_steps=1)
    w = C.synth_weights(cfg, seed=6)
    data = np.random.default_rng(2).integers(0, 64, size=170).astype(np.uint8)
    res = compress_full_sha_incremental(w, data, cfg=cfg, device=DEV, progress=False, verify_decode=True)
    assert res["sha256_ok"] and res["roundtrip_ok"] and res["retrain_count"] == 4
    dec = decompress_full_sha_incremental(w, res["payload"], len(data), cfg=cfg, device=DEV, progress=False)
    assert dec["decoded_sha256"] == res["sha256"]


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_step_reads_the_updated_weights(golden, tensor_cores):
    """After a full-parameter boundary the decode step runs the updated model:
    its logits equal the oracle's on the arena's weights (both linear paths;
    the CUDA-core path reads the arena as dense groups)."""
    from altxs_b200.replenish import ReplenishTTT, state_from_arena
    from oracle.model import OracleModel
    from tests.test_gpu_step import _run_logits

    g = golden("replenish.npz")
    cfg, w0, _ = replenish_case(g, "xm")
    dm = _model(cfg, w0, tensor_cores)
    ttt = ReplenishTTT(dm, n_total=100)
    prefix = torch.as_tensor(g["arr"].astype(np.int32), device=DEV)
    for end in (24, 48):
        ttt.boundary(prefix, end)
    torch.cuda.synchronize()
    st = state_from_arena(dm)
    assert float(np.abs(st["qo_bank"] - w0["qo_bank"]).max()) > 1e-4  # the update moved the weights
    om = OracleReplenish(cfg, st).model()
    toks = g["arr"][:30]
    got = _run_logits(dm, [toks])[0]
    ref_st = om.new_stream()
    ref = np.stack([om.step(ref_st, int(t)).numpy() for t in toks])
    assert float(np.abs(got - ref).max()) < 2e-3
    del OracleModel
