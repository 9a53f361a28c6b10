"""Full-parameter replenish update of one stream's model (B200 kernels).

The reference's production update (altxs ``src/xsa_ttt/compress.py``
``online_retrain`` with ``retrain_mode="replenish"``, :816-1073) trains every
weight of the model at each segment boundary: cross-entropy on a chunk of
``online_retrain_every`` symbols with the preceding ``block_size`` symbols as
context (``chunk_tf_train_loss``, :128-170), global-norm clip, AdamW.  With
``ttt_replenish_xm_k >= 2`` a boundary is a Forward-XM step instead
(``_xm_replenish_boundary``, :611-718): one AdamW step on the previous chunk
gives ΔW; the candidates W0 + s·ΔW (s in 0.5, 1, 2 and 4 while the stream is
short) are scored by the mean cross-entropy on held-out probe chunks
(``_xm_probe_ce``, :523-583) and the best is kept.

Device work goes through the C-ABI: ``altxs_full_loss_grad`` (forward, loss
and the gradient of every parameter), ``altxs_adamw``, ``altxs_params_axpy``
(ΔW and the candidates), ``altxs_params_anchor`` and ``altxs_split_params``
(the step's planes).  The schedule below — warmup, anneal, ramp, replay
draws, candidate and probe windows — is host arithmetic on a few integers,
restated from compress.py:122-126, 323-482 and config.py:447-473.  Every
choice depends only on (config, position) and on device results that the
encoder and the decoder compute bit-identically, so both sides stay in
lockstep.
"""

from __future__ import annotations

import ctypes as C
import math

import numpy as np
import torch

from . import _lib
from .config import ModelConfig
from .engine import DeviceModel, _stream_handle


# ---- host schedule (compress.py:122-126, 323-360, 363-396, 448-520) ------------

def chunk_ctx_start(chunk_start: int, block_size: int) -> tuple[int, int]:
    """(p0, ctx_start) of a chunk: the first coded position and its context start."""
    p0 = 1 if chunk_start == 0 else int(chunk_start)
    return p0, max(0, p0 - int(block_size))


def steps_at(cfg: ModelConfig, position: int, gate: bool = True) -> int:
    """Steps of the update at ``position`` (_online_steps_at, compress.py:323-341);
    ``gate=False`` for callers that decide the boundaries themselves (streams on
    shifted segment clocks)."""
    every = max(1, int(cfg.online_retrain_every))
    if position > 0 and cfg.ttt_bootstrap_steps > 0 and position == cfg.ttt_bootstrap_symbols:
        return int(cfg.ttt_bootstrap_steps)
    if position <= 0 or (gate and position % every):
        return 0
    steps = int(cfg.online_retrain_steps)
    for entry in str(cfg.ttt_burst_schedule or "").split(","):
        entry = entry.strip()
        if not entry:
            continue
        pos_s, sep, n_s = entry.partition(":")
        if not sep or int(pos_s) <= 0 or int(n_s) <= 0:
            raise ValueError(f"burst entry {entry!r} must be pos:steps with positive values")
        if position - every < int(pos_s) <= position:
            steps = max(steps, int(n_s))
    return steps


def anneal(cfg: ModelConfig, end: int, n_total: int | None) -> float | None:
    if str(cfg.ttt_replenish_anneal).lower() == "linear" and n_total:
        total = int(cfg.ttt_replenish_total_bytes) or int(n_total)
        return max(0.0, 1.0 - float(end) / float(total))
    if cfg.ttt_replenish_lr_half_mb > 0:
        return 2.0 ** (-float(end) / (cfg.ttt_replenish_lr_half_mb * 1e6))
    return None


def lr_at(cfg: ModelConfig, end: int, n_total: int | None) -> float:
    f = anneal(cfg, end, n_total)
    lr = float(cfg.ttt_lora_lr) if f is None else max(float(cfg.ttt_replenish_lr_min), float(cfg.ttt_lora_lr) * f)
    if cfg.ttt_replenish_warmup_steps > 0:
        if max(1, int(end) // max(1, int(cfg.online_retrain_every))) <= cfg.ttt_replenish_warmup_steps:
            return 0.0
    return float(lr)


def candidates(cfg: ModelConfig, end: int) -> list[tuple[int, int, float]]:
    every = max(1, int(cfg.online_retrain_every))
    prev = int(end) - every
    c_end = prev if prev >= 2 else int(end)
    c_start = max(0, c_end - every)
    scales = [0.5, 1.0, 2.0][: min(max(2, int(cfg.ttt_replenish_xm_k)), 3)]
    until = int(cfg.ttt_replenish_xm_4x_until_bytes or 0)
    if until > 0 and int(end) < until and 4.0 not in scales:
        scales.append(4.0)
    return [(c_start, c_end, s) for s in scales]


def probe_windows(cfg: ModelConfig, end: int) -> list[tuple[int, int, int]]:
    """(ctx_start, chunk_end, p0) of the held-out probe chunks, newest first,
    skipping the XM training chunk."""
    every = max(1, int(cfg.online_retrain_every))
    n_probe = max(1, int(cfg.ttt_replenish_xm_probe_chunks))
    prev = int(end) - every
    skip = (max(0, prev - every), prev) if prev >= 2 else (-1, -1)
    out, c_end = [], int(end)
    for _ in range(n_probe + 8):
        if len(out) >= n_probe or c_end < 2:
            break
        c_start = max(0, c_end - every)
        if (c_start, c_end) == skip:
            c_end = c_start
            continue
        p0, ctx = chunk_ctx_start(c_start, cfg.block_size)
        if p0 < c_end and c_end - ctx >= 2:
            out.append((ctx, c_end, p0))
        c_end = c_start
    return out


def window_start(end: int, block_size: int) -> int | None:
    """First index of the "full" mode's window arr[start:end] (its last block_size
    positions, compress.py:301-320), or None when it holds fewer than 2."""
    if end < 2:
        return None
    t = min(int(block_size), int(end) - 1)
    return None if t < 2 else int(end) - t - 1


def replay_window_end(cfg: ModelConfig, end: int, step_index: int) -> int:
    """Older window end for the "full" mode's replay steps (compress.py:343-360)."""
    lo = int(min(end, int(cfg.block_size) + 1))
    if step_index <= 0 or lo >= end:
        return int(end)
    mix = (int(cfg.seed) * 1_000_003 + int(end) * 31) ^ (int(step_index) * 0x9E3779B1)
    return int(np.random.default_rng(mix & 0x7FFF_FFFF_FFFF).integers(lo, int(end) + 1))


def replay_end(cfg: ModelConfig, end: int, step_index: int) -> int:
    every = max(1, int(cfg.online_retrain_every))
    n_chunks = max(1, int(end) // every)
    lo = 1
    if cfg.ttt_replenish_replay_recent_mb > 0:
        lo = max(1, n_chunks - max(1, int(cfg.ttt_replenish_replay_recent_mb * 1e6) // every) + 1)
    mix = (int(cfg.seed) * 1_000_003 + int(end) * 31) ^ (int(step_index) * 0x9E3779B1)
    return int(np.random.default_rng(mix & 0x7FFF_FFFF_FFFF).integers(lo, n_chunks + 1)) * every


# ---- reference state dict <-> parameter arena ------------------------------------

def arena_names(cfg: ModelConfig) -> list[str]:
    L = cfg.num_layers
    names = ["tok_emb.weight", "qo_bank", "kv_bank", "mlp_up_bank", "mlp_down_bank"]
    if cfg.num_skip_weights:
        names += ["skip_weights", "skip_gates"]
    for i in range(L):
        names += [f"blocks.{i}.attn_scale", f"blocks.{i}.mlp_scale", f"blocks.{i}.resid_mix", f"blocks.{i}.attn.q_gain"]
    return names


def state_from_arena(dm: DeviceModel, flat: torch.Tensor | None = None) -> dict[str, np.ndarray]:
    """The arena (or ``flat``, another vector in its layout: a gradient, a
    moment) as reference-named arrays (qo_bank = q then o of each layer,
    kv_bank = k then v; model.py:997-1011)."""
    cfg, L, d, kv = dm.cfg, dm.cfg.num_layers, dm.cfg.model_dim, dm.cfg.kv_dim
    src = dm if flat is None else _ArenaOf(dm, flat)
    a = {k: src.arena(k).detach().cpu().numpy() for k in
         ("emb", "qkv", "o", "up", "down", "q_gain", "attn_scale", "mlp_scale", "resid_mix", "skip_weights",
          "skip_gates", "smear_gate", "smear_lambda", "attn_gate_w", "softcap", "parallel_post", "parallel_resid")}
    qkv = a["qkv"].reshape(L, d + 2 * kv, d)
    out = {
        "tok_emb.weight": a["emb"].reshape(cfg.vocab_size, d),
        "qo_bank": np.concatenate([qkv[:, :d], a["o"].reshape(L, d, d)]),
        "kv_bank": np.concatenate([qkv[:, d:d + kv], qkv[:, d + kv:]]),
        "mlp_up_bank": a["up"].reshape(L, cfg.mlp_hidden, d),
        "mlp_down_bank": a["down"].reshape(L, d, cfg.mlp_hidden),
    }
    if cfg.num_skip_weights:
        out["skip_weights"] = a["skip_weights"].reshape(-1, d)
        out["skip_gates"] = a["skip_gates"].reshape(-1, d)
    for i in range(L):
        out[f"blocks.{i}.attn_scale"] = a["attn_scale"].reshape(L, d)[i]
        out[f"blocks.{i}.mlp_scale"] = a["mlp_scale"].reshape(L, d)[i]
        out[f"blocks.{i}.resid_mix"] = a["resid_mix"].reshape(L, 2, d)[i]
        out[f"blocks.{i}.attn.q_gain"] = a["q_gain"].reshape(L, cfg.num_heads)[i]
        if cfg.sparse_attn_gate_enabled:
            out[f"blocks.{i}.attn.attn_gate_w"] = a["attn_gate_w"].reshape(L, cfg.num_heads, cfg.gate_window)[i]
    if cfg.smear_gate_enabled:  # model.py:1101-1105
        out["smear_gate.weight"] = a["smear_gate"].reshape(1, cfg.gate_window)
        out["smear_lambda"] = a["smear_lambda"].reshape(1)
    if cfg.asym_logit_rescale:
        out["softcap_pos"] = a["softcap"][0].copy()
        out["softcap_neg"] = a["softcap"][1].copy()
    if cfg.parallel_start_layer > 0:
        out["parallel_post_lambdas"] = a["parallel_post"].reshape(L, 2, 2)
        out["parallel_resid_lambdas"] = a["parallel_resid"].reshape(L, 2)
    return out


def arena_slices(dm: DeviceModel, name: str, shape) -> torch.Tensor:
    """Arena view holding the reference tensor ``name`` laid out as ``shape``
    (None where the tensor is not one contiguous segment: qo_bank, kv_bank)."""
    cfg, L, d = dm.cfg, dm.cfg.num_layers, dm.cfg.model_dim
    direct = {"tok_emb.weight": "emb", "mlp_up_bank": "up", "mlp_down_bank": "down", "skip_weights": "skip_weights",
              "skip_gates": "skip_gates", "smear_gate.weight": "smear_gate", "smear_lambda": "smear_lambda",
              "parallel_post_lambdas": "parallel_post", "parallel_resid_lambdas": "parallel_resid"}
    if name in direct:
        return dm.arena(direct[name]).view(*shape)
    if name in ("softcap_pos", "softcap_neg"):
        k = 0 if name == "softcap_pos" else 1
        return dm.arena("softcap")[k: k + 1].view(*shape)
    if name.startswith("blocks."):
        i, field = int(name.split(".")[1]), name.split(".", 2)[2]
        seg = {"attn_scale": "attn_scale", "mlp_scale": "mlp_scale", "resid_mix": "resid_mix",
               "attn.q_gain": "q_gain", "attn.attn_gate_w": "attn_gate_w"}[field]
        per = int(np.prod(shape))
        return dm.arena(seg)[i * per: (i + 1) * per].view(*shape)
    return None


# ---- the boundary driver -------------------------------------------------------

class ReplenishTTT:
    """Boundary update of a ``DeviceModel(full_params=True)``: call with the
    stream's symbols so far (device int32, at least ``end`` of them).  The
    model serves one stream: ``Engine`` codes streams one after another and
    calls ``reset()`` between them."""

    per_stream_model = True
    needs_prefix = True

    def __init__(self, dm: DeviceModel, *, n_total: int | None = None, anchor_masks: dict | None = None):
        cfg = dm.cfg
        if not dm.full_params:
            raise ValueError("replenish needs DeviceModel(full_params=True)")
        if cfg.lora_enabled:
            raise ValueError("the full-parameter updates train the model without adapters")
        if cfg.retrain_mode not in ("replenish", "full"):
            raise ValueError("ReplenishTTT runs retrain_mode 'replenish' or 'full'")
        self.dm, self.cfg = dm, cfg
        self.n_total = n_total
        self.L = _lib.lib()
        every = max(1, int(cfg.online_retrain_every))
        self.n_max = int(cfg.block_size) + every + 1  # longest window: context + chunk
        dm.ensure_rope(self.n_max + 1)
        wsb = int(self.L.altxs_full_workspace_bytes(C.byref(dm.desc), self.n_max))
        if wsb < 0:
            raise ValueError("model shape not supported by the full-parameter kernels")
        dev = dm.device
        self.ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        self.ws_bytes = wsb
        n = dm.layout.total
        self.grad = torch.zeros(n, dtype=torch.float32, device=dev)
        self.m = torch.zeros(n, dtype=torch.float32, device=dev)
        self.v = torch.zeros(n, dtype=torch.float32, device=dev)
        self.partials = torch.zeros(256, dtype=torch.float32, device=dev)
        # slot 0: the training chunk's loss; then one per (candidate, probe window)
        self.loss = torch.zeros(1 + 4 * max(1, int(cfg.ttt_replenish_xm_probe_chunks)), dtype=torch.float32,
                                device=dev)
        self.initial = dm.params_initial
        self.anchor_masks = anchor_masks
        self._anchor = None
        self.w0 = self.delta = self.acc = None
        self.step = 0
        self.bm = self.bv = None  # "full" mode: the burst steps' own AdamW moments
        self.bstep = 0
        self.boundaries = 0
        self.xm_last = None
        self.xm_counts: dict[int, int] = {}
        self.last_loss = float("nan")

    def reset(self) -> None:
        """Back to the shipped weights and a fresh optimizer (a new stream)."""
        self.dm.params.copy_(self.initial)
        self.m.zero_()
        self.v.zero_()
        self.step = 0
        self.bm = self.bv = None
        self.bstep = 0
        self._anchor = None
        self.xm_last = None
        self.dm.refresh()

    # ---- device pieces -----------------------------------------------------------
    def _stream(self) -> int:
        return _stream_handle(self.dm.device)

    def _hp(self, lr: float) -> _lib.TttHparams:
        c = self.cfg
        return _lib.TttHparams(lr=lr, beta1=c.ttt_beta1, beta2=c.ttt_beta2, eps=1e-8,
                               weight_decay=c.ttt_weight_decay, grad_clip=c.grad_clip)

    def _loss_grad(self, prefix: torch.Tensor, ctx: int, c_end: int, first: int, slot: int, grad: bool) -> None:
        toks = prefix[ctx:c_end]
        if not toks.is_contiguous():
            toks = toks.contiguous()
        self._keep = toks
        dm = self.dm
        rc = self.L.altxs_full_loss_grad(
            C.byref(dm.desc), C.byref(dm.weights_struct), C.byref(dm.dense_weights()), toks.data_ptr(),
            int(c_end - ctx), int(first), self.loss[slot:].data_ptr(), self.grad.data_ptr() if grad else None,
            self.ws.data_ptr(), self.ws_bytes, self._stream())
        _lib.check(rc, "altxs_full_loss_grad")

    def _chunk(self, prefix, c_start: int, c_end: int, slot: int, grad: bool) -> bool:
        """Loss (and gradient) of chunk [c_start, c_end); False when it scores nothing."""
        p0, ctx = chunk_ctx_start(c_start, self.cfg.block_size)
        if p0 >= c_end or c_end - ctx < 2:
            return False
        self._loss_grad(prefix, ctx, c_end, max(0, p0 - ctx - 1), slot, grad)
        return True

    def _adam(self, lr: float, grad: torch.Tensor | None = None) -> None:
        self.step += 1
        g = self.grad if grad is None else grad
        hp = self._hp(lr)
        _lib.check(self.L.altxs_adamw(self.dm.layout.total, self.dm.params.data_ptr(), g.data_ptr(),
                                      self.m.data_ptr(), self.v.data_ptr(), C.byref(hp), self.step,
                                      self.partials.data_ptr(), self._stream()), "altxs_adamw")

    def _axpy(self, a: torch.Tensor, s: float, b: torch.Tensor, out: torch.Tensor) -> None:
        _lib.check(self.L.altxs_params_axpy(a.numel(), a.data_ptr(), float(s), b.data_ptr(), out.data_ptr(),
                                            self._stream()), "altxs_params_axpy")

    def _anchor_state(self):
        """Pull masks and the weights at the first boundary (compress.py:399-437)."""
        if not self.anchor_masks:
            return None
        if self._anchor is None:
            pull = torch.zeros_like(self.dm.params)
            n_hit = 0
            for name, lam in self.anchor_masks.items():
                lam = np.asarray(lam, dtype=np.float32)
                view = self._pull_view(pull, name, lam.shape)
                if view is None:
                    continue
                view.copy_(torch.from_numpy(lam * np.float32(self.cfg.ttt_replenish_anchor_rate)))
                n_hit += 1
            self._anchor = (self.dm.params.detach().clone(), pull) if n_hit else ()
        return self._anchor or None

    def _pull_view(self, pull: torch.Tensor, name: str, shape):
        """The part of ``pull`` (arena layout) that the reference tensor ``name`` occupies."""
        cfg, dm = self.cfg, self.dm
        L, d, kv = cfg.num_layers, cfg.model_dim, cfg.kv_dim
        lay = dm.layout
        qn = d + 2 * kv
        if name in ("qo_bank", "kv_bank"):
            want = (2 * L, d, d) if name == "qo_bank" else (2 * L, kv, d)
            if tuple(shape) != want:
                return None
            qkv = pull[lay.qkv: lay.qkv + L * qn * d].view(L, qn, d)
            if name == "qo_bank":
                return _Pair(qkv[:, :d], pull[lay.o: lay.o + L * d * d].view(L, d, d))
            return _Pair(qkv[:, d:d + kv], qkv[:, d + kv:])
        try:
            v = arena_slices(_ArenaOf(dm, pull), name, shape)
        except (KeyError, RuntimeError, ValueError):
            return None
        return v if v is not None and tuple(v.shape) == tuple(shape) else None

    def _apply_anchor(self, anchor) -> None:
        if anchor:
            w0, pull = anchor
            _lib.check(self.L.altxs_params_anchor(pull.numel(), self.dm.params.data_ptr(), w0.data_ptr(),
                                                  pull.data_ptr(), self._stream()), "altxs_params_anchor")

    # ---- one boundary ----------------------------------------------------------
    def __call__(self, b, rows, end: int, prefix: torch.Tensor | None = None) -> None:
        """``prefix``: the stream's symbols on the device, [>= end] or [>= end][1]."""
        if prefix is None:
            raise ValueError("replenish needs the stream's symbols (prefix)")
        if prefix.dim() == 2:
            prefix = prefix[:, 0].contiguous()
        self.boundary(prefix, int(end))

    def _burst_adam(self) -> None:
        """One step of the burst optimizer (lr, betas and decay ttt_burst_*)."""
        c = self.cfg
        if self.bm is None:
            self.bm, self.bv = torch.zeros_like(self.m), torch.zeros_like(self.v)
        self.bstep += 1
        hp = _lib.TttHparams(lr=c.ttt_burst_lr, beta1=c.ttt_burst_beta1, beta2=c.ttt_burst_beta2, eps=1e-8,
                             weight_decay=c.ttt_burst_weight_decay, grad_clip=c.grad_clip)
        _lib.check(self.L.altxs_adamw(self.dm.layout.total, self.dm.params.data_ptr(), self.grad.data_ptr(),
                                      self.bm.data_ptr(), self.bv.data_ptr(), C.byref(hp), self.bstep,
                                      self.partials.data_ptr(), self._stream()), "altxs_adamw")

    def _full(self, prefix: torch.Tensor, end: int) -> None:
        """The reference's "full" mode (online_retrain without its replenish
        branch, compress.py:923-1146): mean CE over the last block window; replay
        windows after the first step; at burst boundaries every step runs on the
        burst optimizer and walks the segment boundaries oldest -> newest, the
        last one on the newest window."""
        cfg = self.cfg
        every = max(1, int(cfg.online_retrain_every))
        steps = steps_at(cfg, end)
        if steps == 0 or window_start(end, cfg.block_size) is None:
            return
        replay = bool(cfg.online_retrain_replay) and steps > 1
        burst = steps > max(1, int(cfg.online_retrain_steps)) and bool(str(cfg.ttt_burst_schedule or ""))
        bounds = list(range(every, int(end) + 1, every)) or [int(end)]
        cur = int(end)
        self.boundaries += 1
        for si in range(steps):
            if burst:
                end_k = int(end) if si == steps - 1 else bounds[si % len(bounds)]
                if end_k != cur and window_start(end_k, cfg.block_size) is not None:
                    cur = end_k
            elif replay and si > 0:
                end_k = replay_window_end(cfg, end, si)
                if window_start(end_k, cfg.block_size) is not None:
                    cur = end_k
            self._loss_grad(prefix, window_start(cur, cfg.block_size), cur, 0, 0, True)
            if burst:
                self._burst_adam()
            else:
                self._adam(float(cfg.ttt_lora_lr))
            self.dm.refresh()  # the next step's forward reads the tensor-core planes

    def boundary(self, prefix: torch.Tensor, end: int) -> None:
        cfg = self.cfg
        if cfg.retrain_mode == "full":
            self._full(prefix, int(end))
            return
        every = max(1, int(cfg.online_retrain_every))
        steps = steps_at(cfg, end)
        if steps == 0 or end < 2 or min(int(cfg.block_size), end - 1) < 2:
            return
        if cfg.ttt_replenish_ramp > 0:
            steps = min(steps, 1 + max(0, end // every - 1) // cfg.ttt_replenish_ramp)
        f = anneal(cfg, end, self.n_total)
        if f is not None:
            steps = min(steps, max(max(1, cfg.ttt_replenish_steps_min), int(math.ceil(steps * f))))
        lr = lr_at(cfg, end, self.n_total)
        replay = bool(cfg.online_retrain_replay) and steps > 1
        anchor = self._anchor_state()
        self.boundaries += 1
        if cfg.ttt_replenish_xm_k >= 2 and lr > 0.0:
            self._xm(prefix, end, lr, anchor)
        else:
            accum = steps > 1 and bool(cfg.ttt_replenish_accum)
            if accum:
                if self.acc is None:
                    self.acc = torch.zeros_like(self.grad)
                self.acc.zero_()
            for si in range(steps):
                c_end = replay_end(cfg, end, si) if (replay and si < steps - 1) else end - (steps - 1 - si) * every
                if c_end < 2:
                    continue
                # a chunk that scores nothing leaves no gradient: the reference's
                # optimizer then skips the step (unreachable for c_end >= 2)
                if not self._chunk(prefix, max(0, c_end - every), c_end, 0, True):
                    continue
                if accum:
                    self._axpy(self.acc, 1.0 / steps, self.grad, self.acc)
                    if si == steps - 1:
                        self._adam(lr, self.acc)
                        self._apply_anchor(anchor)
                        self.dm.refresh()
                    continue
                step_lr = lr
                if cfg.ttt_replenish_replay_lr_scale != 1.0 and si < steps - 1:
                    step_lr = lr * cfg.ttt_replenish_replay_lr_scale
                self._adam(step_lr)
                self._apply_anchor(anchor)
                self.dm.refresh()  # the next step's forward reads the tensor-core planes

    def _xm(self, prefix: torch.Tensor, end: int, lr: float, anchor) -> None:
        cands = candidates(self.cfg, end)
        c_start, c_end, _ = cands[0]
        p = self.dm.params
        if self.w0 is None:
            self.w0, self.delta = torch.empty_like(p), torch.empty_like(p)
        self.w0.copy_(p)
        if self._chunk(prefix, c_start, c_end, 0, True):
            self._adam(lr)
        self._axpy(p, -1.0, self.w0, self.delta)  # ΔW at scale 1
        wins = probe_windows(self.cfg, end)
        for k, (_, _, s) in enumerate(cands):
            self._axpy(self.w0, s, self.delta, p)
            self._apply_anchor(anchor)
            self.dm.refresh()
            for j, (ctx, ce, p0) in enumerate(wins):
                self._loss_grad(prefix, ctx, ce, max(0, p0 - ctx - 1), 1 + k * len(wins) + j, False)
        got = self.loss[1: 1 + len(cands) * len(wins)].cpu().numpy().astype(np.float64).reshape(len(cands), -1) \
            if wins else np.zeros((len(cands), 0))
        # mean over the probe windows, summed in order like the reference's Python loop
        scores = []
        for k in range(len(cands)):
            tot = 0.0
            for j in range(len(wins)):
                tot += float(np.float32(got[k, j]))
            scores.append(tot / max(1, len(wins)) if wins else 0.0)
        best = min(range(len(scores)), key=lambda i: (scores[i], i))
        self._axpy(self.w0, cands[best][2], self.delta, p)
        self._apply_anchor(anchor)
        self.dm.refresh()
        self.xm_last = {"end": int(end), "chosen": int(best), "scores": scores, "candidates": cands}
        self.xm_counts[best] = self.xm_counts.get(best, 0) + 1


class _Pair:
    """Two arena views that together hold one reference bank (q|o or k|v halves)."""

    def __init__(self, a: torch.Tensor, b: torch.Tensor):
        self.a, self.b = a, b
        self.shape = (a.shape[0] + b.shape[0],) + tuple(a.shape[1:])

    def copy_(self, src: torch.Tensor) -> None:
        n = self.a.shape[0]
        self.a.copy_(src[:n].to(self.a.device))
        self.b.copy_(src[n:].to(self.b.device))


class _ArenaOf:
    """``DeviceModel.arena`` over another tensor in the same layout."""

    def __init__(self, dm: DeviceModel, t: torch.Tensor):
        self.cfg, self._dm, self._t = dm.cfg, dm, t

    def arena(self, name: str) -> torch.Tensor:
        v = self._dm.arena(name)
        off = v.data_ptr() - self._dm.params.data_ptr()
        return self._t[off // 4: off // 4 + v.numel()]
