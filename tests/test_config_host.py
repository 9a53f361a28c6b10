"""Host-side configuration logic (no GPU): the adapter layout of the reference's
TTTLoRA (order, MLP adapters, one slot per layer application), the adapter
mask handed to the kernels, and which reference configurations the engine
accepts or refuses."""

from __future__ import annotations

import pytest

from altxs_b200.config import ModelConfig
from altxs_b200.lora import init_lora_A, lora_shapes

BASE = dict(vocab_size=256, num_layers=4, model_dim=64, num_heads=4, num_kv_heads=2, mlp_mult=2.0, rope_dims=8,
            block_size=16, online_retrain_every=32, seed=5)


def test_lora_layout_follows_ttt_lora_parameter_order():
    """lm, then q, v, k, mlp, o over the slots (ttt_lora.py:67-105 registration order)."""
    cfg = ModelConfig(**BASE, ttt_lora_rank=4, ttt_k_lora=True, ttt_o_lora=True, ttt_mlp_lora=True)
    names = list(lora_shapes(cfg))
    L = cfg.num_layers
    assert names == ["lm"] + [f"q{i}" for i in range(L)] + [f"v{i}" for i in range(L)] + \
        [f"k{i}" for i in range(L)] + [f"mlp{i}" for i in range(L)] + [f"o{i}" for i in range(L)]
    shapes = lora_shapes(cfg)
    d, kv, r = cfg.model_dim, cfg.kv_dim, cfg.ttt_lora_rank
    assert shapes["lm"] == ((r, d), (cfg.vocab_size, r))
    assert shapes["v0"] == ((r, d), (kv, r))
    assert shapes["mlp0"] == ((r, d), (d, r))


def test_lora_slots_follow_the_depth_loop_schedule():
    """With depth loops every application has its own adapters (six slots for
    four layers with one loop over layers 1-2)."""
    cfg = ModelConfig(**BASE, ttt_lora_rank=4, num_loops=1, loop_start=1, loop_end=2)
    assert cfg.layer_schedule == ([0, 1, 2], [1, 2, 3])
    assert [k for k in lora_shapes(cfg) if k.startswith("q")] == [f"q{s}" for s in range(6)]
    A = init_lora_A(cfg)
    assert list(A) == list(lora_shapes(cfg)) and A["q5"].shape == (4, cfg.model_dim)


def test_adapter_mask_bits():
    from altxs_b200.engine import lora_mask

    cfg = ModelConfig(**BASE, ttt_lora_rank=4, ttt_k_lora=False, ttt_o_lora=True, ttt_mlp_lora=True,
                      ttt_o_lora_on_y=True)
    assert lora_mask(cfg) == 1 | 4 | 16 | 8 | 32 | 64
    cfg = ModelConfig(**BASE, ttt_lora_rank=4, ttt_k_lora=True, ttt_o_lora=False, ttt_o_lora_on_y=True)
    assert lora_mask(cfg) == 1 | 4 | 16 | 2  # o on y means nothing without the o adapter
    assert lora_mask(ModelConfig(**BASE, retrain_mode="none")) == 0


def test_rank_range_and_lane_rule():
    ModelConfig(**BASE, ttt_lora_rank=128).validate()
    with pytest.raises(ValueError):
        ModelConfig(**BASE, ttt_lora_rank=129).validate()
    # full-parameter updates: once a decoder application runs two lanes, every later one must
    ok = ModelConfig(**BASE, retrain_mode="replenish", parallel_start_layer=2)
    ok.validate()
    bad = ModelConfig(**{**BASE, "num_layers": 6}, retrain_mode="full", num_loops=1, loop_start=2, loop_end=4,
                      parallel_start_layer=4)
    assert bad.layer_schedule[1] == [4, 2, 3, 4, 5]
    with pytest.raises(ValueError):
        bad.validate()


@pytest.mark.parametrize("mode", ["lora", "replenish", "full"])
def test_reference_cfg_keeps_the_retrain_mode_with_motifs(mode):
    """A reference config with motifs keeps its retrain mode (every update
    computes them); the options no profile uses stay refused."""
    ref = dict(BASE, retrain_mode=mode, smear_gate_enabled=True, xsa_last_n=2, sparse_attn_gate_enabled=True,
               asym_logit_rescale=True, num_loops=1, loop_start=1, loop_end=2, parallel_start_layer=3,
               ttt_lora_rank=8, ttt_mlp_lora=True)
    cfg = ModelConfig.from_reference_cfg(ref)
    assert cfg.retrain_mode == mode and cfg.motifs
    cfg.validate()
    for opt in ("attn_out_gate_enabled", "gated_attn_enabled", "rope_yarn"):
        with pytest.raises(ValueError):
            ModelConfig.from_reference_cfg(dict(ref, **{opt: True}))
    with pytest.raises(ValueError):
        ModelConfig.from_reference_cfg(dict(ref, tie_embeddings=False))
