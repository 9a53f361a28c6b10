"""CPU restatement of the reference's full-parameter replenish update.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA replenish path.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline may
import it; the product never routes through it.

Follows altxs ``src/xsa_ttt/compress.py``:
  * ``_chunk_ctx_start`` / ``chunk_tf_train_loss``  :122-170  (CE on one chunk,
    the preceding ``block_size`` symbols as context, positions from 0)
  * ``_online_steps_at``, ``_replay_window_end``     :323-360
  * ``_scheduled_replenish_lr``                     :363-396
  * ``_replenish_anchor_state`` / ``_apply_...``    :399-445  (w -= pull (w - w0))
  * ``_xm_candidates``, ``_xm_probe_windows``        :448-520
  * ``_xm_probe_ce``                                :523-583
  * ``_xm_replenish_boundary`` (shared-window path) :611-718
  * ``online_retrain`` replenish branch             :816-1073 (ramp, anneal taper,
    replay draws, walk-back, XM dispatch)
with the optimizer of ``_init_online_state`` (compress.py:1976-1985): AdamW
over every parameter, lr ``ttt_lora_lr``, betas ``ttt_beta1/2``,
``ttt_weight_decay``, global-norm clip ``grad_clip``; burst steps from
``parse_burst_schedule`` (config.py:454-473).

The "full" mode (the reference's default ``retrain_mode``; ``online_retrain``
:923-1146 without the replenish branch) is restated too: the window loss of
the last ``block_size`` symbols (``_window_xy`` :301-320, ``GPT.forward``
model.py:1502-1510), replay windows (``_replay_window_end`` :343-360) and
burst steps on a second AdamW (``ttt_burst_*``) that walk the segment
boundaries oldest -> newest.

The serial XM fallback (compress.py:721-802) is unreachable: every candidate
trains on the same window, which always holds >= 2 symbols past ``end >= 2``.
Pinned against the reference's own ``online_retrain`` (tests/golden/replenish.npz).
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from altxs_b200.config import ModelConfig
from oracle.model import OracleModel, OracleWeights

# reference names of the five weight banks (model.py:997-1011)
BANKS = ("tok_emb.weight", "qo_bank", "kv_bank", "mlp_up_bank", "mlp_down_bank")
# model-level motif parameters (the per-block sparse gate is blocks.{i}.attn.attn_gate_w)
MOTIF_PARAMS = ("smear_gate.weight", "smear_lambda", "softcap_pos", "softcap_neg", "parallel_post_lambdas",
                "parallel_resid_lambdas")


def chunk_ctx_start(chunk_start: int, block_size: int) -> tuple[int, int]:
    p0 = 1 if chunk_start == 0 else int(chunk_start)
    return p0, max(0, p0 - int(block_size))


def online_steps_at(position: int, cfg: ModelConfig, every: int) -> int:
    if position > 0 and cfg.ttt_bootstrap_steps > 0 and position == cfg.ttt_bootstrap_symbols:
        return int(cfg.ttt_bootstrap_steps)
    if position <= 0 or every <= 0 or position % every:
        return 0
    steps = int(cfg.online_retrain_steps)
    for part in str(cfg.ttt_burst_schedule or "").split(","):
        if part.strip():
            pos, _, n = part.strip().partition(":")
            if position - every < int(pos) <= position:
                steps = max(steps, int(n))
    return steps


def anneal_factor(cfg: ModelConfig, end: int, n_total: int | None):
    mode = str(cfg.ttt_replenish_anneal).lower()
    if mode == "linear" and n_total:
        total = int(cfg.ttt_replenish_total_bytes) or int(n_total)
        return max(0.0, 1.0 - float(end) / float(total))
    if cfg.ttt_replenish_lr_half_mb > 0:
        return 2.0 ** (-float(end) / (cfg.ttt_replenish_lr_half_mb * 1e6))
    return None


def scheduled_lr(cfg: ModelConfig, end: int, n_total: int | None) -> float:
    lr = float(cfg.ttt_lora_lr)
    factor = anneal_factor(cfg, end, n_total)
    if factor is not None:
        lr = max(float(cfg.ttt_replenish_lr_min), float(cfg.ttt_lora_lr) * factor)
    if cfg.ttt_replenish_warmup_steps > 0:
        b = max(1, int(end) // max(1, int(cfg.online_retrain_every)))
        if b <= cfg.ttt_replenish_warmup_steps:
            return 0.0
    return float(lr)


def xm_candidates(cfg: ModelConfig, end: int) -> list[tuple[int, int, float]]:
    every = max(1, int(cfg.online_retrain_every))
    prev_end = int(end) - every
    if prev_end >= 2:
        c_end, c_start = prev_end, max(0, prev_end - every)
    else:
        c_end, c_start = int(end), max(0, int(end) - every)
    chosen = [0.5, 1.0, 2.0][: min(max(2, int(cfg.ttt_replenish_xm_k)), 3)]
    until = int(cfg.ttt_replenish_xm_4x_until_bytes or 0)
    if until > 0 and int(end) < until and 4.0 not in chosen:
        chosen.append(4.0)
    return [(c_start, c_end, float(s)) for s in chosen]


def xm_probe_windows(end: int, every: int, n_probe: int, block_size: int) -> list[tuple[int, int, int]]:
    every = max(1, int(every))
    prev_end = int(end) - every
    if prev_end >= 2:
        train_end, train_start = prev_end, max(0, prev_end - every)
    else:
        train_end = train_start = -1
    out = []
    c_end = int(end)
    for _ in range(max(1, n_probe) + 8):
        if len(out) >= max(1, n_probe) or c_end < 2:
            break
        c_start = max(0, c_end - every)
        if c_start == train_start and c_end == train_end:
            c_end = c_start
            continue
        p0, ctx = chunk_ctx_start(c_start, block_size)
        if p0 < c_end and c_end - ctx >= 2:
            out.append((ctx, c_end, p0))
        c_end = c_start
    return out


def window_start(end: int, block_size: int) -> int | None:
    """First index of the last-block window ``arr[start:end]`` (x = [:-1], y = [1:])."""
    if end < 2:
        return None
    t = min(int(block_size), end - 1)
    return None if t < 2 else end - t - 1


def replay_window_end(end: int, step_index: int, seed: int, block_size: int) -> int:
    lo = int(min(end, int(block_size) + 1))
    if step_index <= 0 or lo >= end:
        return int(end)
    mix = (int(seed) * 1_000_003 + int(end) * 31) ^ (int(step_index) * 0x9E3779B1)
    return int(np.random.default_rng(mix & 0x7FFF_FFFF_FFFF).integers(lo, int(end) + 1))


def replay_chunk_end(cfg: ModelConfig, seed: int, end: int, step_index: int) -> int:
    """Chunk end drawn for replay step ``step_index`` (compress.py:1012-1037)."""
    every = max(1, int(cfg.online_retrain_every))
    n_chunks = max(1, int(end) // every)
    lo = 1
    if cfg.ttt_replenish_replay_recent_mb > 0:
        span = max(1, int(cfg.ttt_replenish_replay_recent_mb * 1e6) // every)
        lo = max(1, n_chunks - span + 1)
    mix = (int(seed) * 1_000_003 + int(end) * 31) ^ (int(step_index) * 0x9E3779B1)
    rng = np.random.default_rng(mix & 0x7FFF_FFFF_FFFF)
    return int(rng.integers(lo, n_chunks + 1)) * every


class OracleReplenish:
    """Every parameter of one stream's model + its AdamW state (torch, CPU)."""

    def __init__(self, cfg: ModelConfig, state: dict, anchor_masks: dict | None = None):
        """``state``: reference-named fp32 arrays (a GPT state dict)."""
        self.cfg = cfg
        L = cfg.num_layers
        t = lambda a: torch.tensor(np.asarray(a, dtype=np.float32)).requires_grad_(True)  # noqa: E731
        self.p = {k: t(state[k]) for k in BANKS}
        for name in ("skip_weights", "skip_gates"):
            if name in state and np.asarray(state[name]).size:
                self.p[name] = t(state[name])
        for i in range(L):
            for k in ("attn_scale", "mlp_scale", "resid_mix", "attn.q_gain"):
                self.p[f"blocks.{i}.{k}"] = t(state[f"blocks.{i}.{k}"])
            if cfg.sparse_attn_gate_enabled:
                self.p[f"blocks.{i}.attn.attn_gate_w"] = t(state[f"blocks.{i}.attn.attn_gate_w"])
        # motif parameters (model.py:753-758, 994-996, 1092-1105), trained like every
        # other when their motif is on; the reference model always holds the
        # parallel lambdas, which get no gradient (AdamW skips them) with the lanes off
        on = {"smear_gate.weight": cfg.smear_gate_enabled, "smear_lambda": cfg.smear_gate_enabled,
              "softcap_pos": cfg.asym_logit_rescale, "softcap_neg": cfg.asym_logit_rescale,
              "parallel_post_lambdas": cfg.parallel_start_layer > 0,
              "parallel_resid_lambdas": cfg.parallel_start_layer > 0}
        for name in MOTIF_PARAMS:
            if on[name]:
                self.p[name] = t(state[name])
        self.params = list(self.p.values())
        self.opt = torch.optim.AdamW(self.params, lr=cfg.ttt_lora_lr, betas=(cfg.ttt_beta1, cfg.ttt_beta2),
                                     weight_decay=cfg.ttt_weight_decay)
        self.anchor_masks = anchor_masks
        self.anchor = None
        self.xm_last = None
        self.burst_opt = None

    # ---- forward ---------------------------------------------------------------
    def weights(self) -> OracleWeights:
        cfg, p, L = self.cfg, self.p, self.cfg.num_layers
        small = {
            "q_gain": torch.stack([p[f"blocks.{i}.attn.q_gain"] for i in range(L)]),
            "attn_scale": torch.stack([p[f"blocks.{i}.attn_scale"] for i in range(L)]),
            "mlp_scale": torch.stack([p[f"blocks.{i}.mlp_scale"] for i in range(L)]),
            "resid_mix": torch.stack([p[f"blocks.{i}.resid_mix"] for i in range(L)]),
            "skip_weights": p.get("skip_weights", torch.zeros(0, cfg.model_dim)),
            "skip_gates": p.get("skip_gates", torch.zeros(0, cfg.model_dim)),
        }
        if "smear_gate.weight" in p:
            small["smear_gate"] = p["smear_gate.weight"].reshape(-1)
            small["smear_lambda"] = p["smear_lambda"].reshape(1)
        if "blocks.0.attn.attn_gate_w" in p:
            small["attn_gate_w"] = torch.stack([p[f"blocks.{i}.attn.attn_gate_w"] for i in range(L)])
        if "softcap_pos" in p:
            small["softcap"] = torch.stack([p["softcap_pos"].reshape(()), p["softcap_neg"].reshape(())])
        if "parallel_post_lambdas" in p:
            small["parallel_post"] = p["parallel_post_lambdas"]
            small["parallel_resid"] = p["parallel_resid_lambdas"]
        return OracleWeights(
            cfg=cfg, emb=p["tok_emb.weight"],
            q=[p["qo_bank"][i] for i in range(L)], o=[p["qo_bank"][L + i] for i in range(L)],
            k=[p["kv_bank"][i] for i in range(L)], v=[p["kv_bank"][L + i] for i in range(L)],
            up=[p["mlp_up_bank"][i] for i in range(L)], down=[p["mlp_down_bank"][i] for i in range(L)],
            small=small,
        )

    def model(self) -> OracleModel:
        return OracleModel(self.weights())

    def window_ce(self, ids: np.ndarray, first: int) -> torch.Tensor | None:
        """Mean CE of ids[1:] from positions first.. of the forward over ids[:-1]."""
        ids = torch.as_tensor(np.asarray(ids, dtype=np.int64))
        x, y = ids[:-1], ids[1:]
        if y[first:].numel() == 0:
            return None
        logits = self.model().window_logits(x, None)
        return F.cross_entropy(logits[first:].float(), y[first:], reduction="mean")

    def chunk_loss(self, arr: np.ndarray, c_start: int, c_end: int) -> torch.Tensor | None:
        """Mean CE on symbols [c_start, c_end) with the preceding block as context."""
        p0, ctx = chunk_ctx_start(c_start, self.cfg.block_size)
        if p0 >= c_end or c_end - ctx < 2:
            return None
        return self.window_ce(arr[ctx:c_end], max(0, p0 - ctx - 1))

    @torch.no_grad()
    def probe_ce(self, arr: np.ndarray, end: int) -> float:
        cfg = self.cfg
        wins = xm_probe_windows(end, cfg.online_retrain_every, cfg.ttt_replenish_xm_probe_chunks, cfg.block_size)
        if not wins:
            return 0.0
        total = 0.0
        for ctx, c_end, p0 in wins:
            ce = self.window_ce(arr[ctx:c_end], max(0, p0 - ctx - 1))
            if ce is not None:
                total += float(ce)
        return total / max(1, len(wins))

    # ---- optimizer pieces --------------------------------------------------------
    def _step(self, loss: torch.Tensor) -> None:
        loss.backward()
        torch.nn.utils.clip_grad_norm_(self.params, self.cfg.grad_clip)
        self.opt.step()

    def _anchor_state(self):
        if not self.anchor_masks:
            return None
        if self.anchor is None:  # weights at the first boundary (compress.py:399-437)
            ent = []
            for name, lam in self.anchor_masks.items():
                p = self.p.get(name)
                if p is None or tuple(p.shape) != tuple(np.shape(lam)):
                    continue
                pull = torch.as_tensor(np.asarray(lam, dtype=np.float32)) * float(self.cfg.ttt_replenish_anchor_rate)
                ent.append((p, p.detach().clone(), pull))
            self.anchor = ent
        return self.anchor

    @torch.no_grad()
    def _apply_anchor(self, anchor) -> None:
        for p, w0, pull in anchor or ():
            p.sub_((p - w0) * pull)

    def _set_lr(self, lr: float) -> None:
        for g in self.opt.param_groups:
            g["lr"] = float(lr)

    # ---- one boundary ----------------------------------------------------------
    def boundary(self, arr: np.ndarray, end: int, n_total: int | None = None) -> float:
        """Reference ``online_retrain`` in replenish (or full) mode at position ``end``."""
        cfg = self.cfg
        if cfg.retrain_mode == "full":
            return self._full(arr, end)
        every = max(1, int(cfg.online_retrain_every))
        steps = online_steps_at(end, cfg, every)
        if steps == 0 or end < 2 or min(int(cfg.block_size), end - 1) < 2:
            return float("nan")
        if cfg.ttt_replenish_ramp > 0:
            steps = min(steps, 1 + max(0, int(end) // every - 1) // cfg.ttt_replenish_ramp)
        factor = anneal_factor(cfg, end, n_total)
        if factor is not None:
            steps = min(steps, max(max(1, cfg.ttt_replenish_steps_min), int(math.ceil(steps * factor))))
        lr_eff = scheduled_lr(cfg, end, n_total)
        self._set_lr(lr_eff)
        replay = bool(cfg.online_retrain_replay) and steps > 1
        anchor = self._anchor_state()
        if cfg.ttt_replenish_xm_k >= 2 and lr_eff > 0.0:
            return self._xm(arr, end, lr_eff, anchor)
        accum = steps > 1 and bool(cfg.ttt_replenish_accum)
        last = float("nan")
        if accum:
            self.opt.zero_grad(set_to_none=True)
        for si in range(steps):
            if replay and si < steps - 1:
                c_end = replay_chunk_end(cfg, cfg.seed, end, si)
            else:
                c_end = int(end) - (steps - 1 - si) * every
            if c_end < 2:
                continue
            c_start = max(0, c_end - every)
            if not accum:
                self.opt.zero_grad(set_to_none=True)
            with torch.enable_grad():
                loss = self.chunk_loss(arr, c_start, c_end)
                if loss is None:
                    loss = torch.zeros((), requires_grad=True)
                if accum:
                    (loss / float(steps)).backward()
                    if si == steps - 1:
                        torch.nn.utils.clip_grad_norm_(self.params, cfg.grad_clip)
                        self.opt.step()
                        self.opt.zero_grad(set_to_none=True)
                        self._apply_anchor(anchor)
                    last = float(loss.detach())
                    continue
                if cfg.ttt_replenish_replay_lr_scale != 1.0:
                    self._set_lr(lr_eff if si == steps - 1 else lr_eff * cfg.ttt_replenish_replay_lr_scale)
                self._step(loss)
            self._apply_anchor(anchor)
            last = float(loss.detach())
        return last

    def _full(self, arr: np.ndarray, end: int) -> float:
        cfg = self.cfg
        every = max(1, int(cfg.online_retrain_every))
        steps = online_steps_at(end, cfg, every)
        if steps == 0 or end < 2 or window_start(end, cfg.block_size) is None:
            return float("nan")
        replay = bool(cfg.online_retrain_replay) and steps > 1
        is_burst = steps > max(1, int(cfg.online_retrain_steps)) and bool(str(cfg.ttt_burst_schedule or ""))
        if is_burst and self.burst_opt is None:
            self.burst_opt = torch.optim.AdamW(self.params, lr=cfg.ttt_burst_lr,
                                               betas=(cfg.ttt_burst_beta1, cfg.ttt_burst_beta2),
                                               weight_decay=cfg.ttt_burst_weight_decay)
        bounds = list(range(every, int(end) + 1, every)) or [int(end)]
        cur = int(end)
        last = float("nan")
        for si in range(steps):
            if is_burst:
                end_k = int(end) if si == steps - 1 else bounds[si % len(bounds)]
                if end_k != cur and window_start(end_k, cfg.block_size) is not None:
                    cur = end_k
            elif replay and si > 0:
                end_k = replay_window_end(end, si, cfg.seed, cfg.block_size)
                if window_start(end_k, cfg.block_size) is not None:
                    cur = end_k
            opt = self.burst_opt if is_burst else self.opt
            opt.zero_grad(set_to_none=True)
            with torch.enable_grad():
                loss = self.window_ce(arr[window_start(cur, cfg.block_size): cur], 0)
                loss.backward()
            torch.nn.utils.clip_grad_norm_(self.params, cfg.grad_clip)
            opt.step()
            last = float(loss.detach())
        return last

    def _xm(self, arr: np.ndarray, end: int, lr_eff: float, anchor) -> float:
        cands = xm_candidates(self.cfg, end)
        c_start, c_end, _ = cands[0]
        w0 = [p.detach().clone() for p in self.params]
        self._set_lr(lr_eff)
        self.opt.zero_grad(set_to_none=True)
        with torch.enable_grad():
            loss = self.chunk_loss(arr, c_start, c_end)
            if loss is None:
                loss = torch.zeros((), requires_grad=True)
            self._step(loss)
        last = float(loss.detach())
        with torch.no_grad():
            delta = [p.detach() - w for p, w in zip(self.params, w0)]

        def materialize(s: float) -> None:
            with torch.no_grad():
                for p, w, d in zip(self.params, w0, delta):
                    p.copy_(w + float(s) * d)
            self._apply_anchor(anchor)

        scores = []
        for _, _, s in cands:
            materialize(s)
            scores.append(self.probe_ce(arr, end))
        best = min(range(len(scores)), key=lambda i: (scores[i], i))
        materialize(cands[best][2])
        self._set_lr(lr_eff * cands[best][2])
        self.xm_last = {"end": int(end), "chosen": int(best), "scores": scores, "candidates": cands}
        return last

    def state(self) -> dict:
        return {k: v.detach().numpy().copy() for k, v in self.p.items()}
