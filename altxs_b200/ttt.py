"""Test-time LoRA update at segment boundaries (host side).

At every boundary ``end`` (a positive multiple of ``online_retrain_every``)
each stream trains its adapters for ``_online_steps_at`` AdamW steps
(``online_retrain_steps``, bootstrap and burst positions; compress.py:323-341),
the first on its own last window:
``x = s[end-T-1 : end-1]``, ``y = s[end-T : end]`` with ``T = min(block_size,
end-1)`` and no update when ``T < 2`` (reference ``_window_xy`` and
``should_online_retrain_at``, altxs src/xsa_ttt/compress.py:301-320,
config.py:447-451); with ``online_retrain_replay`` the later steps train on
older windows drawn by ``_replay_window_end`` (compress.py:343-360).  Encoder
and decoder call this at the same boundaries on the same symbols, so their
adapters stay bit-identical.  The newest window is read from the device ring
of coded symbols that the step kernel maintains; replay windows from the
stream's symbols, which the engine passes as ``prefix``.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .engine import DeviceModel, StreamBatch, _stream_handle


class LoraTTT:
    needs_prefix = True  # replay steps read windows older than the ring

    def __init__(self, dm: DeviceModel, *, dense_base: bool = True):
        self.dm = dm
        # the tensor-core path reads the bf16 planes; the dense fp32 copy serves the CUDA-core path
        self.dense = dm.dense_weights() if dense_base and not dm.tensor_cores else None
        cfg = dm.cfg
        if not cfg.lora_enabled:
            raise ValueError("test-time update needs retrain_mode='lora' and a positive rank")
        self.hp = _lib.TttHparams(lr=cfg.ttt_lora_lr, beta1=cfg.ttt_beta1, beta2=cfg.ttt_beta2, eps=1e-8,
                                  weight_decay=cfg.ttt_weight_decay, grad_clip=cfg.grad_clip)
        self.t_max = int(cfg.ctx)
        self.ws_bytes = int(_lib.lib().altxs_ttt_workspace_bytes(C.byref(dm.desc), self.t_max))
        if self.ws_bytes < 0:
            raise ValueError("model shape not supported by the update kernels")
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dm.device)
        self.loss = torch.zeros(1, dtype=torch.float32, device=dm.device)
        self._state: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        self.steps: dict[int, dict[int, int]] = {}
        self.ce_history: list[float] = []
        self.record_loss = False

    def _moments(self, b: StreamBatch) -> tuple[torch.Tensor, torch.Tensor]:
        key = id(b)
        if key not in self._state:
            z = torch.zeros_like(b.lora)
            self._state[key] = (z, torch.zeros_like(b.lora))
            self.steps[key] = {}
        return self._state[key]

    def __call__(self, b: StreamBatch, rows, end: int, prefix: torch.Tensor | None = None) -> None:
        """``prefix``: the streams' symbols on the device, [>= end][n] (row r's
        symbols in column r); needed only when replay steps run."""
        from .replenish import replay_window_end, steps_at, window_start

        if b.hist is None or b.lora is None:
            raise RuntimeError("the batch was built without a symbol ring or adapters")
        cfg = self.dm.cfg
        end = int(end)
        n_steps = steps_at(cfg, end, gate=False)  # the caller decides where boundaries are
        if n_steps == 0 or window_start(end, self.t_max) is None:
            return
        replay = bool(cfg.online_retrain_replay) and n_steps > 1
        if replay and prefix is None:
            raise RuntimeError("replay steps need the streams' symbols (prefix)")
        # window end of every step: the newest, then the replay draws (a draw too
        # short for a window keeps the previous one, as the reference does)
        ends, cur = [], end
        for si in range(n_steps):
            if replay and si > 0:
                e = replay_window_end(cfg, end, si)
                if window_start(e, self.t_max) is not None:
                    cur = e
            ends.append(cur)
        m, v = self._moments(b)
        steps = self.steps[id(b)]
        dev = self.dm.device
        L = _lib.lib()
        for r in rows:
            for e in ends:
                s0 = window_start(e, self.t_max)
                T = e - s0 - 1
                if e == end:  # the newest window is in the ring
                    idx = torch.arange(s0, e, device=dev) % b.hist_len
                    window = b.hist[r].index_select(0, idx).contiguous()
                else:
                    window = prefix[s0:e, r].to(torch.int32).contiguous()
                steps[r] = steps.get(r, 0) + 1
                rc = L.altxs_ttt_update(
                    C.byref(self.dm.desc), C.byref(self.dm.weights_struct),
                    C.byref(self.dense) if self.dense is not None else None, C.byref(self.hp), window.data_ptr(), T,
                    b.lora[r].data_ptr(), m[r].data_ptr(), v[r].data_ptr(), steps[r], self.loss.data_ptr(),
                    self.ws.data_ptr(), self.ws_bytes, _stream_handle(dev))
                _lib.check(rc, "altxs_ttt_update")
                if self.record_loss:
                    self.ce_history.append(float(self.loss.item()))
