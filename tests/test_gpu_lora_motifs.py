"""Test-time LoRA on a model with the reference motifs (one adapter slot per
layer application, MLP adapters, adapters inside the parallel lanes) on the
B200 kernels: the step with adapters against the oracle, the update against
the reference's own online_retrain (golden), encode -> decode lockstep."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from altxs_b200 import codec as C
from altxs_b200.config import ModelConfig
from oracle.model import OracleModel, OracleWeights
from tests.test_gpu_motifs import BASE, CASES, _logits_mode
from tests.test_gpu_step import _lora_vec
from tests.test_oracle_golden import motif_case

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
LORA = dict(retrain_mode="lora", ttt_lora_rank=8, ttt_k_lora=True, ttt_o_lora=True, ttt_mlp_lora=True)


def _cfg(name: str, **over) -> ModelConfig:
    kw = dict(BASE)
    kw.update(CASES[name])
    kw.update(LORA)
    kw.update(over)
    return ModelConfig(**kw)


def _weights(cfg, seed=9):
    w = C.synth_weights(cfg, seed=seed)
    rng = np.random.default_rng(seed)
    s = w.small
    s["smear_gate"] = rng.normal(0, 0.5, s["smear_gate"].shape).astype(np.float32)
    s["smear_lambda"] = np.array([0.7], dtype=np.float32)
    s["attn_gate_w"] = rng.normal(0, 0.5, s["attn_gate_w"].shape).astype(np.float32)
    s["softcap"] = np.array([12.0, 20.0], dtype=np.float32)
    s["parallel_post"] = (s["parallel_post"] + rng.normal(0, 0.1, s["parallel_post"].shape)).astype(np.float32)
    s["parallel_resid"] = (s["parallel_resid"] + rng.normal(0, 0.1, s["parallel_resid"].shape)).astype(np.float32)
    return w


@pytest.mark.parametrize("tensor_cores", [True, False])
@pytest.mark.parametrize("name,o_on_y", [("all", False), ("all", True), ("loop", False), ("par_mean", True)])
def test_motif_step_with_adapters_matches_oracle(name, o_on_y, tensor_cores):
    """The decode step of a motif model with random adapters on every slot
    (q/k/v/o/MLP per layer application, lm head): logits within 2e-3 of the
    oracle, past the window."""
    from altxs_b200.engine import DeviceModel

    cfg = _cfg(name, ttt_o_lora_on_y=o_on_y)
    w = _weights(cfg)
    dm = DeviceModel(w, DEV, tensor_cores=tensor_cores)
    vec, lo = _lora_vec(cfg, np.random.default_rng(2))
    toks = np.random.default_rng(5).integers(0, cfg.vocab_size, size=cfg.block_size + 7)
    b_lora = torch.as_tensor(vec, device=DEV)
    got = _logits_mode(dm, [toks], lora=b_lora)[0]
    om = OracleModel(OracleWeights.from_model_weights(w))
    st = om.new_stream()
    ref = np.stack([om.step(st, int(t), lo).numpy() for t in toks])
    err = float(np.abs(got - ref).max())
    assert err < 2e-3, err


@pytest.mark.parametrize("tensor_cores", [False, True])
def test_motif_lora_update_matches_reference(golden, tensor_cores):
    """LoraTTT on the reference's motif model (depth loop active: six adapter
    slots for four layers), two steps per boundary with replay, against the
    reference's online_retrain in lora mode: every boundary's loss, and the
    adapters in units of an Adam step."""
    from altxs_b200.engine import StreamBatch
    from altxs_b200.lora import lora_shapes
    from altxs_b200.ttt import LoraTTT

    from altxs_b200.engine import DeviceModel

    g = golden("motif_retrain.npz")
    cfg, w0 = motif_case(g, "m_lora")
    dm = DeviceModel(C.dense_weights(cfg, {k: np.asarray(v, np.float32) for k, v in w0.items()}), DEV,
                     tensor_cores=tensor_cores)
    names = {"lm": "lm_head_lora"}
    for sl in range(cfg.num_virtual_layers):
        for t, mod in (("q", "q_loras"), ("k", "k_loras"), ("v", "v_loras"), ("o", "o_loras"), ("mlp", "mlp_loras")):
            names[f"{t}{sl}"] = f"{mod}.{sl}"

    def arena(part):
        return np.concatenate(sum([[g[f"m_lora/{part}/{names[k]}.A"].reshape(-1),
                                    g[f"m_lora/{part}/{names[k]}.B"].reshape(-1)] for k in lora_shapes(cfg)], []))

    ttt = LoraTTT(dm)
    b = StreamBatch(dm, 1, words_per_stream=8, hist_len=cfg.ctx + 2)
    assert np.array_equal(b.lora[0].cpu().numpy(), arena("init"))
    arr = g["arr"].astype(np.int32)
    prefix = torch.as_tensor(arr[:, None].copy(), device=DEV)
    diffs = []
    for end in (24, 48, 72, 96):
        pos = torch.arange(max(0, end - b.hist_len), end, device=DEV)
        b.hist[0].index_copy_(0, pos % b.hist_len, prefix[pos, 0])
        ttt(b, [0], end, prefix=prefix)
        diffs.append(abs(float(ttt.loss.item()) - float(g[f"m_lora/{end}/loss"])))
    # the first boundary pins the model; later ones carry the earlier steps' drift
    assert diffs[0] < (2e-4 if tensor_cores else 2e-5), diffs
    assert max(diffs) < (1e-3 if tensor_cores else 1e-4), diffs
    lr = cfg.ttt_lora_lr
    diff = np.abs(b.lora[0].cpu().numpy() - arena("final"))
    # fp32 agrees to a few percent of a step everywhere; the tensor cores' 2^-16
    # products flip the signs of some near-zero gradients over the eight steps,
    # and Adam (beta1 = 0) turns each into part of a step: 99.9 % of entries
    # within half a step, every entry within one (measured worst 0.78 lr)
    frac = 0.5 if tensor_cores else 0.1
    assert (diff <= frac * lr).mean() > 0.999, ((diff > frac * lr).sum(), diff.size)
    assert diff.max() < (1.0 if tensor_cores else 0.1) * lr, diff.max() / lr


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_motif_lora_round_trip(tensor_cores):
    """Encode -> decode with every motif on and LoRA updates at each boundary."""
    from altxs_b200.engine import DeviceModel, Engine
    from altxs_b200.ttt import LoraTTT

    cfg = _cfg("all", block_size=24, online_retrain_every=40, online_retrain_steps=2, ttt_lora_lr=3e-3)
    dm = DeviceModel(_weights(cfg, seed=4), DEV, tensor_cores=tensor_cores)
    rng = np.random.default_rng(3)
    streams = [rng.integers(0, cfg.vocab_size, size=k).astype(np.int32) for k in (130, 97)]
    enc = Engine(dm, ttt=LoraTTT(dm)).encode(streams)
    dec = Engine(dm, ttt=LoraTTT(dm)).decode([r.payload for r in enc], [len(s) for s in streams])
    for s, d in zip(streams, dec):
        assert np.array_equal(s, d)
    plain = Engine(dm).encode(streams)
    assert any(a.segments != b.segments for a, b in zip(enc, plain))
