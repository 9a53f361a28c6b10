"""The device test-time LoRA update against the torch oracle (and the reference)."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from altxs_b200 import codec as C_
from altxs_b200.config import ModelConfig
from oracle.model import OracleModel, OracleTTT, OracleWeights

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")

SMALL = dict(
    vocab_size=512, num_layers=3, model_dim=128, num_heads=4, num_kv_heads=2,
    mlp_mult=4.0, rope_dims=16, block_size=32, online_retrain_every=64, seed=11,
    ttt_lora_rank=4, ttt_lora_lr=1e-3, ttt_k_lora=True, ttt_o_lora=True,
)


def _device_update(dm, lora_vec, window, steps=1, dense=True):
    from altxs_b200 import _lib

    L = _lib.lib()
    cfg = dm.cfg
    hp = _lib.TttHparams(lr=cfg.ttt_lora_lr, beta1=cfg.ttt_beta1, beta2=cfg.ttt_beta2, eps=1e-8,
                         weight_decay=cfg.ttt_weight_decay, grad_clip=cfg.grad_clip)
    T = len(window) - 1
    wsb = L.altxs_ttt_workspace_bytes(C.byref(dm.desc), T)
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
    p = torch.as_tensor(lora_vec, device=DEV).clone()
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    tok = torch.as_tensor(np.asarray(window, np.int32), device=DEV)
    loss = torch.zeros(1, device=DEV)
    losses = []
    for s in range(1, steps + 1):
        dw = C.byref(dm.dense_weights()) if dense else None
        rc = L.altxs_ttt_update(C.byref(dm.desc), C.byref(dm.weights_struct), dw, C.byref(hp), tok.data_ptr(), T,
                                p.data_ptr(), m.data_ptr(), v.data_ptr(), s, loss.data_ptr(), ws.data_ptr(), wsb,
                                torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        losses.append(float(loss.item()))
    return p.cpu().numpy(), losses


def _arena(lora, cfg):
    from altxs_b200.lora import lora_shapes

    out = []
    for name in lora_shapes(cfg):
        out += [lora.A[name].detach().numpy().reshape(-1), lora.B[name].detach().numpy().reshape(-1)]
    return np.concatenate(out)


@pytest.mark.parametrize("path", ["tensor_cores", "dense", "packed"])
def test_ttt_update_matches_oracle(golden, path):
    """The update on the tensor cores, on CUDA cores from a dense fp32 copy of
    the base, and on CUDA cores from the packed codes."""
    from altxs_b200.engine import DeviceModel

    g = golden("lora_small.npz")
    cfg = ModelConfig(**SMALL)
    w = C_.synth_weights(cfg, seed=7)
    dm = DeviceModel(w, DEV, tensor_cores=path == "tensor_cores")
    dense = path == "dense"
    om = OracleModel(OracleWeights.from_model_weights(w))
    ttt = OracleTTT(om)
    vec0 = _arena(ttt.lora, cfg)
    arr, end = g["arr"], int(g["end"])
    t = min(cfg.block_size, end - 1)
    window = arr[end - t - 1: end]
    got, losses = _device_update(dm, vec0, window, steps=2, dense=dense)
    ref_losses = [ttt.update(arr, end) for _ in range(2)]
    np.testing.assert_allclose(losses, ref_losses, rtol=2e-5)
    np.testing.assert_allclose(losses, g["losses"], rtol=2e-5)  # the reference itself
    ref = _arena(ttt.lora, cfg)
    diff = np.abs(got - ref)
    # Adam's first steps move each entry by about lr*sign(grad): entries whose
    # gradient is ~0 may differ by up to 2*lr; everything else agrees closely
    assert (diff <= 1e-5).mean() > 0.999, (diff.max(), (diff > 1e-5).sum())
    assert diff.max() <= 2.1 * cfg.ttt_lora_lr


def test_ttt_update_is_deterministic():
    from altxs_b200.engine import DeviceModel
    from altxs_b200.lora import init_lora_A, lora_shapes

    cfg = ModelConfig(**SMALL)
    dm = DeviceModel(C_.synth_weights(cfg, seed=3), DEV)
    A = init_lora_A(cfg)
    vec = np.concatenate(sum([[A[k].reshape(-1), np.zeros(s[1][0] * s[1][1], np.float32)]
                              for k, s in lora_shapes(cfg).items()], []))
    window = np.random.default_rng(0).integers(0, cfg.vocab_size, size=cfg.block_size + 1)
    a, la = _device_update(dm, vec, window, steps=3)
    b, lb = _device_update(dm, vec, window, steps=3)
    assert la == lb
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("n_streams", [1, 3])
def test_engine_roundtrip_with_ttt(n_streams):
    """Encode -> decode stays bit-exact through several test-time updates."""
    from altxs_b200.engine import DeviceModel, Engine
    from altxs_b200.synth import zipf_markov
    from altxs_b200.ttt import LoraTTT

    cfg = ModelConfig(**SMALL)
    dm = DeviceModel(C_.synth_weights(cfg, seed=9), DEV)
    lens = [260, 130, 65][:n_streams]
    src = zipf_markov(max(lens), cfg.vocab_size, np.arange(n_streams) + 40)
    streams = [src[i, : lens[i]] for i in range(n_streams)]
    enc_ttt = LoraTTT(dm)
    enc = Engine(dm, ttt=enc_ttt).encode(streams)
    dec = Engine(dm, ttt=LoraTTT(dm)).decode([r.payload for r in enc], lens)
    for s, d in zip(streams, dec):
        assert np.array_equal(s, d)
    # the adapters moved (updates happened)
    no = Engine(dm).encode(streams)
    assert any(a.segments != b.segments for a, b in zip(enc, no))


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_lora_steps_with_replay_match_reference(golden, tensor_cores):
    """LoraTTT with three steps per boundary (replay windows after the first,
    read from the stream's symbols) against the reference's own online_retrain
    in lora mode: the adapters after two boundaries."""
    from altxs_b200.engine import DeviceModel, StreamBatch
    from altxs_b200.lora import lora_shapes
    from altxs_b200.ttt import LoraTTT

    g = golden("lora_steps.npz")
    cfg = ModelConfig(**{**SMALL, "online_retrain_steps": 3, "online_retrain_replay": True})
    dm = DeviceModel(C_.synth_weights(cfg, seed=7), DEV, tensor_cores=tensor_cores)
    ttt = LoraTTT(dm)
    b = StreamBatch(dm, 1, words_per_stream=8, hist_len=cfg.ctx + 2)
    arr = g["arr"].astype(np.int32)
    prefix = torch.as_tensor(arr[:, None].copy(), device=DEV)
    every = cfg.online_retrain_every
    for end in (every, 2 * every):
        pos = torch.arange(max(0, end - b.hist_len), end, device=DEV)  # the ring holds the last hist_len symbols
        b.hist[0].index_copy_(0, pos % b.hist_len, prefix[pos, 0])
        ttt(b, [0], end, prefix=prefix)
    torch.cuda.synchronize()
    ref = []
    names = {"lm": "lm_head_lora"}
    for i in range(cfg.num_layers):
        for t in ("q", "k", "v", "o"):
            names[f"{t}{i}"] = f"{t}_loras.{i}"
    for name in lora_shapes(cfg):
        ref += [g[f"final/{names[name]}.A"].reshape(-1), g[f"final/{names[name]}.B"].reshape(-1)]
    ref = np.concatenate(ref)
    got = b.lora[0].cpu().numpy()
    # Adam steps of lr per entry: agreement within a small fraction of one step
    err = float(np.abs(got - ref).max())
    assert err < (0.3 if tensor_cores else 0.05) * cfg.ttt_lora_lr, err
