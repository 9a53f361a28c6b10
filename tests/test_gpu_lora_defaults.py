"""The reference's default LoRA set on the B200 kernels: rank 80, q/v/o + MLP
+ lm_head adapters (k off), the o adapter on the block's normed input or on
the attention output (ttt_o_lora_on_y).  The step with trained adapters
against the oracle, the update against the reference's own online_retrain
(golden), and encode -> decode lockstep."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from altxs_b200 import codec as C_
from altxs_b200.config import ModelConfig
from oracle.model import OracleModel, OracleWeights
from tests.test_gpu_step import _lora_vec, _run_logits
from tests.test_gpu_ttt import SMALL as TTT_SMALL
from tests.test_oracle_golden import SMALL, lora_ref_names

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
CASES = ["base", "o_on_y"]


def _cfg(g, case) -> ModelConfig:
    return ModelConfig(**{**SMALL, **json.loads(bytes(g[f"{case}/over"]))})


def _golden_arena(g, case, cfg, part="final"):
    from altxs_b200.lora import lora_shapes

    names = lora_ref_names(cfg)
    out = []
    for name in lora_shapes(cfg):
        out += [g[f"{case}/{part}/{names[name]}.A"].reshape(-1), g[f"{case}/{part}/{names[name]}.B"].reshape(-1)]
    return np.concatenate(out)


@pytest.mark.parametrize("tensor_cores", [True, False])
@pytest.mark.parametrize("case", CASES)
def test_lora_defaults_update_matches_reference(golden, case, tensor_cores):
    """LoraTTT with the default adapter set, two steps per boundary (replay on
    the second), against the reference's online_retrain: every boundary's loss,
    and the adapters after two boundaries."""
    from altxs_b200.engine import DeviceModel, StreamBatch
    from altxs_b200.ttt import LoraTTT

    g = golden("lora_defaults.npz")
    cfg = _cfg(g, case)
    dm = DeviceModel(C_.synth_weights(cfg, seed=7), DEV, tensor_cores=tensor_cores)
    assert dm.lora_floats == len(_golden_arena(g, case, cfg, "init"))
    ttt = LoraTTT(dm)
    b = StreamBatch(dm, 1, words_per_stream=8, hist_len=cfg.ctx + 2)
    assert np.array_equal(b.lora[0].cpu().numpy(), _golden_arena(g, case, cfg, "init"))
    arr = g["arr"].astype(np.int32)
    prefix = torch.as_tensor(arr[:, None].copy(), device=DEV)
    every = cfg.online_retrain_every
    for end in (every, 2 * every):
        pos = torch.arange(max(0, end - b.hist_len), end, device=DEV)
        b.hist[0].index_copy_(0, pos % b.hist_len, prefix[pos, 0])
        ttt(b, [0], end, prefix=prefix)
        # the loss of the boundary's last step, as the reference's online_retrain returns it
        loss = float(ttt.loss.item())
        assert abs(loss - float(g[f"{case}/{end}/loss"])) < (2e-4 if tensor_cores else 2e-5), (end, loss)
    torch.cuda.synchronize()
    lr = cfg.ttt_lora_lr
    diff = np.abs(b.lora[0].cpu().numpy() - _golden_arena(g, case, cfg))
    # From the second step on every A entry gets gradient through B != 0; a few
    # dozen of the rank-80 A entries have gradients near zero whose sign follows
    # summation order, and Adam with beta1 = 0 turns a sign into a step of up to
    # lr * sqrt((1 - beta2^t) / (1 - beta2)) at step t (1, 1.41, 1.72, 1.98 lr over
    # the four steps).  The bulk agrees to a tenth of a step; the worst entry stays
    # inside the largest displacement four steps can make.
    assert (diff <= 0.1 * lr).mean() > 0.999, ((diff > 0.1 * lr).sum(), diff.size)
    assert diff.max() < 6.2 * lr, diff.max()


@pytest.mark.parametrize("tensor_cores", [True, False])
@pytest.mark.parametrize("o_on_y", [False, True])
def test_step_with_mlp_and_o_adapters_matches_oracle(tensor_cores, o_on_y):
    """The decode step with random (non-zero) rank-80 adapters on q/v/o/MLP and
    the LM head: logits within 2e-3 of the oracle across the sliding window."""
    from altxs_b200.engine import DeviceModel

    cfg = ModelConfig(**{**TTT_SMALL, "ttt_lora_rank": 80, "ttt_k_lora": False, "ttt_mlp_lora": True,
                         "ttt_o_lora_on_y": o_on_y})
    w = C_.synth_weights(cfg, seed=5)
    dm = DeviceModel(w, DEV, tensor_cores=tensor_cores)
    vec, lo = _lora_vec(cfg, np.random.default_rng(4))
    toks = np.random.default_rng(6).integers(0, cfg.vocab_size, size=cfg.block_size + 9)
    got = _run_logits(dm, [toks], lora_vec=vec)[0]
    om = OracleModel(OracleWeights.from_model_weights(w))
    st = om.new_stream()
    ref = np.stack([om.step(st, int(t), lo).numpy() for t in toks])
    err = float(np.abs(got - ref).max())
    assert err < 2e-3, err


@pytest.mark.parametrize("tensor_cores", [True, False])
def test_engine_round_trip_with_default_adapters(tensor_cores):
    """Encode -> decode through several boundaries with the default adapter set."""
    from altxs_b200.engine import DeviceModel, Engine
    from altxs_b200.ttt import LoraTTT

    cfg = ModelConfig(**{**TTT_SMALL, "ttt_lora_rank": 80, "ttt_k_lora": False, "ttt_mlp_lora": True,
                         "ttt_o_lora_on_y": True, "online_retrain_steps": 2})
    dm = DeviceModel(C_.synth_weights(cfg, seed=9), DEV, tensor_cores=tensor_cores)
    rng = np.random.default_rng(1)
    streams = [rng.integers(0, cfg.vocab_size, size=k).astype(np.int32) for k in (230, 140)]
    enc = Engine(dm, ttt=LoraTTT(dm)).encode(streams)
    dec = Engine(dm, ttt=LoraTTT(dm)).decode([r.payload for r in enc], [len(s) for s in streams])
    for s, d in zip(streams, dec):
        assert np.array_equal(s, d)
    plain = Engine(dm).encode(streams)
    assert any(a.segments != b.segments for a, b in zip(enc, plain))
