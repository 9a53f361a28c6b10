"""Host side of the replenish update: the product's boundary schedule equals
the oracle's restatement of the reference (pinned by the golden) on a sweep of
positions and configurations."""

from __future__ import annotations

import itertools

from altxs_b200 import replenish as R
from altxs_b200.config import ModelConfig
from oracle import replenish as O


def _cfgs():
    for every, block, k, probes, until, warm, half, recent, burst in itertools.product(
            (24, 4096), (16, 2048), (0, 2, 3), (1, 2), (0, 100_000), (0, 3), (0.0, 0.05), (0.0, 1.0),
            ("", "200:4")):
        yield ModelConfig(num_layers=2, model_dim=64, num_heads=4, num_kv_heads=2, vocab_size=64,
                          retrain_mode="replenish", online_retrain_every=every, block_size=block,
                          ttt_replenish_xm_k=k, ttt_replenish_xm_probe_chunks=probes,
                          ttt_replenish_xm_4x_until_bytes=until, ttt_replenish_warmup_steps=warm,
                          ttt_replenish_lr_half_mb=half, ttt_replenish_replay_recent_mb=recent,
                          ttt_burst_schedule=burst, online_retrain_steps=3, seed=7)


def test_schedule_matches_oracle():
    n = 0
    for cfg in _cfgs():
        e = cfg.online_retrain_every
        for end in (1, 2, e - 1, e, 2 * e, 3 * e, 7 * e, 200, 30 * e):
            assert R.steps_at(cfg, end) == O.online_steps_at(end, cfg, e)
            assert R.lr_at(cfg, end, 50 * e) == O.scheduled_lr(cfg, end, 50 * e)
            assert R.anneal(cfg, end, None) == O.anneal_factor(cfg, end, None)
            if end >= 2:
                assert R.candidates(cfg, end) == O.xm_candidates(cfg, end)
                assert R.probe_windows(cfg, end) == O.xm_probe_windows(
                    end, e, cfg.ttt_replenish_xm_probe_chunks, cfg.block_size)
                for si in range(3):
                    assert R.replay_end(cfg, end, si) == O.replay_chunk_end(cfg, cfg.seed, end, si)
                    assert R.replay_window_end(cfg, end, si) == O.replay_window_end(end, si, cfg.seed,
                                                                                    cfg.block_size)
            assert R.window_start(end, cfg.block_size) == O.window_start(end, cfg.block_size)
            n += 1
    assert n > 1000
