"""Torch fp32 CPU restatement of the altxs GPT step, LoRA and test-time update.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  This is the
floating-point reference the CUDA step is checked against (tolerance-based)
and the CPU baseline that ``bench.py`` times.

Restated from the altxs reference (paths inside that project):
  * embedding + RMSNorm, no smear           src/xsa_ttt/model.py:1536-1549
  * Block.forward (resid_mix, ln_scale,
    attn_scale, mlp_scale)                  src/xsa_ttt/model.py:948-979
  * CausalSelfAttention.forward (QK-RMSNorm,
    partial RoPE, q_gain, SDPA, out proj)   src/xsa_ttt/model.py:770-871
  * Rotary tables / apply_rotary_emb        src/xsa_ttt/model.py:130-205
  * MLP LeakyReLU(0.5)^2                     src/xsa_ttt/model.py:874-882
  * U-Net skips with sigmoid gates (lerp)   src/xsa_ttt/model.py:1395-1436
  * tied logits + tanh softcap              src/xsa_ttt/model.py:1460-1476,1495-1500
  * LoRA deltas (q/k/v/o on the block's
    normed input, lm_head on final hidden)  src/xsa_ttt/ttt_lora.py:22-56,124-179,258-350
  * CE + clip 1.0 + AdamW step              src/xsa_ttt/ttt_lora.py:353-374,
                                            src/xsa_ttt/compress.py:1104-1137
  * LoRA A init order and seed              src/xsa_ttt/ttt_lora.py:67-105,
                                            src/xsa_ttt/compress.py:1965-1974
  * training window (last block_size)       src/xsa_ttt/compress.py:301-320
  * motifs: smear gate                       src/xsa_ttt/model.py:1350-1362
            XSA, sparse attention gate       src/xsa_ttt/model.py:760-768, 845-862
            depth-loop layer schedule        src/xsa_ttt/model.py:1064-1077, 1377-1436
            parallel lanes                   src/xsa_ttt/model.py:1293-1348, 1404-1443
            asymmetric softcap               src/xsa_ttt/model.py:1478-1500

Context semantics.  The reference re-prefills a context at each segment
boundary; this engine instead keeps a sliding window of the last
``block_size`` tokens (ring buffer, RoPE at absolute positions).  The step
below implements exactly that rule.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch
import torch.nn.functional as F

from altxs_b200.config import ModelConfig
from altxs_b200.lora import init_lora_A, lora_shapes, rope_tables


@dataclass
class OracleWeights:
    cfg: ModelConfig
    emb: torch.Tensor
    q: list
    k: list
    v: list
    o: list
    up: list
    down: list
    small: dict

    @classmethod
    def from_model_weights(cls, w) -> "OracleWeights":
        d = w.dense()
        L = w.cfg.num_layers
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))  # noqa: E731
        return cls(
            cfg=w.cfg,
            emb=t(d["tok_emb.weight"]),
            q=[t(d["qo_bank"][i]) for i in range(L)],
            o=[t(d["qo_bank"][L + i]) for i in range(L)],
            k=[t(d["kv_bank"][i]) for i in range(L)],
            v=[t(d["kv_bank"][L + i]) for i in range(L)],
            up=[t(d["mlp_up_bank"][i]) for i in range(L)],
            down=[t(d["mlp_down_bank"][i]) for i in range(L)],
            small={k2: t(v2) for k2, v2 in w.small.items()},
        )


@dataclass
class OracleLoRA:
    """Per-stream adapters: name -> (A [r, in], B [out, r]) per layer."""

    A: dict = field(default_factory=dict)
    B: dict = field(default_factory=dict)

    @classmethod
    def init(cls, cfg: ModelConfig) -> "OracleLoRA":
        A = {k: torch.from_numpy(v.copy()) for k, v in init_lora_A(cfg).items()}
        B = {k: torch.zeros(shp[1]) for k, shp in lora_shapes(cfg).items()}
        return cls(A=A, B=B)

    def delta(self, name: str, x: torch.Tensor, scale: float) -> torch.Tensor:
        # (x @ A.T @ B.T) * scale   (ttt_lora.py:54-56)
        return (x @ self.A[name].T @ self.B[name].T) * scale

    def params(self, cfg: ModelConfig) -> list:
        """Parameter order of the reference TTTLoRA.parameters()."""
        out = []
        for name in lora_shapes(cfg):
            out += [self.A[name], self.B[name]]
        return out


def _rms(x: torch.Tensor) -> torch.Tensor:
    return F.rms_norm(x, (x.size(-1),))


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rd: int) -> torch.Tensor:
    # apply_rotary_emb (model.py:195-205); x [..., T, H, D], cos/sin [T, 1, rd/2]
    x_rope, x_pass = x[..., :rd], x[..., rd:]
    half = rd // 2
    x1, x2 = x_rope[..., :half], x_rope[..., half:]
    x_rope = torch.cat((x1 * cos + x2 * sin, x1 * -sin + x2 * cos), dim=-1)
    return torch.cat((x_rope, x_pass), dim=-1)


class OracleModel:
    """Sliding-window stepper + teacher-forced window forward."""

    def __init__(self, w: OracleWeights):
        self.w = w
        cfg = w.cfg
        self.cfg = cfg
        self.cos, self.sin = (torch.from_numpy(a) for a in rope_tables(cfg, 1 << 12))
        # optional rounding of every stored K/V value (a callable on fp32
        # tensors): emulates a KV-cache storage format in precision studies
        self.kv_round = None

    def _tables(self, pos: torch.Tensor):
        need = int(pos.max()) + 1
        if need > self.cos.shape[0]:
            n = 1 << max(12, (need - 1).bit_length())
            self.cos, self.sin = (torch.from_numpy(a) for a in rope_tables(self.cfg, n))
        return self.cos[pos][:, None, :], self.sin[pos][:, None, :]

    # ---- one block over rows x [T, d] with queries at positions qpos ---------
    def _attn(self, i, n, x_pos, kv_prefix, lora, causal, slot=None):
        """Attention of layer i; adapters of slot ``slot`` (the application index)."""
        s = i if slot is None else slot
        cfg, w = self.cfg, self.w
        H, Hkv, D, rd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.rope_dims
        T = n.shape[0]
        q = n @ w.q[i].T
        k = n @ w.k[i].T
        v = n @ w.v[i].T
        if lora is not None:
            sc = cfg.lora_scale
            q = q + lora.delta(f"q{s}", n, sc)
            if f"k{s}" in lora.A:
                k = k + lora.delta(f"k{s}", n, sc)
            v = v + lora.delta(f"v{s}", n, sc)
        q = _rms(q.view(T, H, D))
        k = _rms(k.view(T, Hkv, D))
        v = v.view(T, Hkv, D)
        cos, sin = self._tables(x_pos)
        q = _rope(q, cos, sin, rd)
        k = _rope(k, cos, sin, rd)
        q = q * w.small["q_gain"][i][None, :, None]
        if self.kv_round is not None:
            k, v = self.kv_round(k), self.kv_round(v)
        v_new = v
        if kv_prefix is not None:
            pk, pv = kv_prefix
            k_all = torch.cat([pk, k], 0)
            v_all = torch.cat([pv, v], 0)
        else:
            k_all, v_all = k, v
        rep = H // Hkv
        ke = k_all.repeat_interleave(rep, dim=1)
        ve = v_all.repeat_interleave(rep, dim=1)
        y = F.scaled_dot_product_attention(
            q.transpose(0, 1)[None], ke.transpose(0, 1)[None], ve.transpose(0, 1)[None],
            is_causal=causal,
        )[0].transpose(0, 1)
        if cfg.xsa_last_n > 0 and i >= cfg.num_layers - cfg.xsa_last_n:
            # remove each head's component along its own token's value direction
            vn = F.normalize(v_new, dim=-1)[:, :, None, :]  # [T, Hkv, 1, D]
            yg = y.reshape(T, Hkv, rep, D)
            y = (yg - (yg * vn).sum(-1, keepdim=True) * vn).reshape(T, H, D)
        if cfg.sparse_attn_gate_enabled:
            gw = cfg.gate_window
            g = torch.sigmoid(cfg.sparse_attn_gate_scale * (n[:, :gw] @ w.small["attn_gate_w"][i].T))  # [T, H]
            y = y * g[:, :, None]
        y = y.reshape(T, H * D)
        out = y @ w.o[i].T
        if lora is not None and f"o{s}" in lora.A:  # ttt_lora.py:168-170
            out = out + lora.delta(f"o{s}", y if cfg.ttt_o_lora_on_y else n, cfg.lora_scale)
        return out, (k, v)

    def _block(self, i, x, x0, x_pos, kv_prefix, lora, causal, slot=None):
        cfg, sm = self.cfg, self.w.small
        s = i if slot is None else slot
        ln = 1.0 / math.sqrt(i + 1) if cfg.ln_scale else 1.0
        mix = sm["resid_mix"][i]
        x_in = mix[0][None, :] * x + mix[1][None, :] * x0
        n = _rms(x_in) * ln
        attn_out, kv_new = self._attn(i, n, x_pos, kv_prefix, lora, causal, s)
        x_out = x_in + sm["attn_scale"][i][None, :] * attn_out
        mlp_n = _rms(x_out) * ln
        h = F.leaky_relu(mlp_n @ self.w.up[i].T, negative_slope=0.5).square()
        mlp_out = h @ self.w.down[i].T
        if lora is not None and f"mlp{s}" in lora.A:  # ttt_lora.py:171-174
            mlp_out = mlp_out + lora.delta(f"mlp{s}", mlp_n, cfg.lora_scale)
        x_out = x_out + sm["mlp_scale"][i][None, :] * mlp_out
        return x_out, kv_new

    def _parallel_block(self, i, lane0, lane1, x0, x_pos, kv_prefix, causal, lora=None, slot=None):
        """Two-lane block (model.py:1293-1351; with adapters ttt_lora.py:181-250)."""
        cfg, sm = self.cfg, self.w.small
        s = i if slot is None else slot
        ln = 1.0 / math.sqrt(i + 1) if cfg.ln_scale else 1.0
        mix = sm["resid_mix"][i]
        n = _rms(mix[0][None, :] * lane0 + mix[1][None, :] * x0) * ln
        attn_out, kv_new = self._attn(i, n, x_pos, kv_prefix, lora, causal, s)
        attn_out = sm["attn_scale"][i][None, :] * attn_out
        mlp_n = _rms(lane1) * ln
        h = F.leaky_relu(mlp_n @ self.w.up[i].T, negative_slope=0.5).square()
        mlp_raw = h @ self.w.down[i].T
        if lora is not None and f"mlp{s}" in lora.A:
            mlp_raw = mlp_raw + lora.delta(f"mlp{s}", mlp_n, cfg.lora_scale)
        mlp_out = sm["mlp_scale"][i][None, :] * mlp_raw
        pr, pp = sm["parallel_resid"][i], sm["parallel_post"][i]
        lane0 = pr[0] * lane0 + pp[0][0] * attn_out + pp[1][0] * mlp_out
        lane1 = pr[1] * lane1 + pp[0][1] * attn_out + pp[1][1] * mlp_out
        return lane0, lane1, kv_new

    def _embed(self, tokens, prev_tok):
        cfg, sm = self.cfg, self.w.small
        raw = self.w.emb[tokens]
        if not cfg.smear_gate_enabled:
            return raw
        prev = torch.cat([self.w.emb[[prev_tok]] if prev_tok is not None else torch.zeros_like(raw[:1]), raw[:-1]])
        g = sm["smear_lambda"][0] * torch.sigmoid(raw[:, : cfg.gate_window] @ sm["smear_gate"])
        return raw + g[:, None] * prev

    def _stack(self, tokens, x_pos, kv_prefixes, lora, causal, prev_tok=None):
        cfg, sm = self.cfg, self.w.small
        x = _rms(self._embed(tokens, prev_tok))
        x0 = x
        enc, dec = cfg.layer_schedule
        skips, new_kv = [], []
        for i in enc:  # the application index is the adapter slot
            x, kv = self._block(i, x, x0, x_pos, kv_prefixes[len(new_kv)], lora, causal, len(new_kv))
            new_kv.append(kv)
            skips.append(x)
        psl = cfg.parallel_start_layer
        lane0 = lane1 = None

        def skip_into(dest, skip_idx):
            if skip_idx < cfg.num_skip_weights and skips:
                scaled = sm["skip_weights"][skip_idx][None, :] * skips.pop()
                if cfg.skip_gates_enabled:
                    return torch.lerp(scaled, dest, torch.sigmoid(sm["skip_gates"][skip_idx])[None, :])
                return dest + scaled
            return dest

        for skip_idx, i in enumerate(dec):
            if psl > 0 and i >= psl:
                if lane0 is None:
                    lane0 = lane1 = x
                lane0 = skip_into(lane0, skip_idx)
                lane0, lane1, kv = self._parallel_block(i, lane0, lane1, x0, x_pos,
                                                        kv_prefixes[len(new_kv)], causal, lora, len(new_kv))
            else:
                x = skip_into(x, skip_idx)
                x, kv = self._block(i, x, x0, x_pos, kv_prefixes[len(new_kv)], lora, causal, len(new_kv))
            new_kv.append(kv)
        if lane0 is not None:
            fl = cfg.parallel_final_lane
            x = lane1 if fl == "mlp" else lane0 if fl == "attn" else 0.5 * (lane0 + lane1)
        h = _rms(x)
        logits = h @ self.w.emb.T
        if lora is not None:
            logits = logits + lora.delta("lm", h, cfg.lora_scale)
        if cfg.asym_logit_rescale:
            sp, sn = sm["softcap"][0], sm["softcap"][1]
            return torch.where(logits >= 0, sp * torch.tanh(logits / sp), sn * torch.tanh(logits / sn)), new_kv
        c = cfg.logit_softcap
        return c * torch.tanh(logits / c), new_kv

    # ---- sliding-window decode ----------------------------------------------
    def new_stream(self):
        return {"pos": 0, "kv": [None] * self.cfg.num_virtual_layers, "prev": None}

    @torch.no_grad()
    def step(self, st, tok: int, lora: OracleLoRA | None = None) -> torch.Tensor:
        """Consume ``tok`` at position ``st['pos']``; return next-symbol logits."""
        cfg = self.cfg
        pos = st["pos"]
        x_pos = torch.tensor([pos])
        keep = cfg.kv_len - 1  # the current key makes the window ``kv_len`` wide
        prefixes = []
        for kv in st["kv"]:
            if kv is None or keep == 0:
                prefixes.append(None)
            else:
                prefixes.append((kv[0][-keep:], kv[1][-keep:]))
        logits, new_kv = self._stack(torch.tensor([tok]), x_pos, prefixes, lora, causal=False,
                                     prev_tok=st.get("prev"))
        st["prev"] = int(tok)
        for i, (k, v) in enumerate(new_kv):
            if prefixes[i] is None:
                st["kv"][i] = (k, v)
            else:
                st["kv"][i] = (torch.cat([prefixes[i][0], k]), torch.cat([prefixes[i][1], v]))
        st["pos"] = pos + 1
        return logits[0]

    @torch.no_grad()
    def prefill(self, st, tokens, lora: OracleLoRA | None = None) -> torch.Tensor:
        """Consume ``tokens`` from an empty stream in one causal pass (the
        last ``ctx-1`` keys are kept); returns the last position's logits."""
        if st["pos"] != 0:
            raise ValueError("prefill starts from an empty stream")
        toks = torch.as_tensor(np.asarray(tokens, dtype=np.int64))
        T = toks.shape[0]
        if T > self.cfg.kv_len:
            raise ValueError("prefill longer than the window is not a sliding-window pass")
        logits, new_kv = self._stack(toks, torch.arange(T), [None] * self.cfg.num_virtual_layers, lora,
                                     causal=True)
        st["kv"] = list(new_kv)
        st["pos"] = T
        st["prev"] = int(toks[-1])
        return logits[-1]

    def reset_segment(self, arr, start: int, lora: OracleLoRA | None = None):
        """Segment-reset context (reference reset_segment + _chunk_ctx_start,
        incremental.py:858-897, compress.py:122-125): a fresh stream holding
        the first n-1 of the last n = min(block_size, start) symbols before
        ``start`` at positions 0..n-2.  Stepping arr[start-1] next gives the
        distribution of symbol ``start``.  Returns the stream."""
        st = self.new_stream()
        n = min(int(self.cfg.block_size), int(start))
        if n > 1:
            self.prefill(st, np.asarray(arr[start - n: start - 1]), lora)
        return st

    # ---- teacher-forced window (training forward) --------------------------
    def window_logits(self, tokens: torch.Tensor, lora: OracleLoRA | None) -> torch.Tensor:
        T = tokens.shape[0]
        logits, _ = self._stack(tokens, torch.arange(T), [None] * self.cfg.num_virtual_layers, lora, causal=True)
        return logits


def window_xy(arr: np.ndarray, end: int, block_size: int):
    """Teacher-forced (x, y) from arr[:end] (compress.py:301-320)."""
    if end < 2:
        return None
    t = min(int(block_size), end - 1)
    start = end - t - 1
    x = np.asarray(arr[start: start + t], dtype=np.int64)
    y = np.asarray(arr[start + 1: start + 1 + t], dtype=np.int64)
    if x.shape[0] < 2:
        return None
    return torch.from_numpy(x), torch.from_numpy(y)


class OracleTTT:
    """LoRA adapters + AdamW state for one stream."""

    def __init__(self, model: OracleModel):
        cfg = model.cfg
        self.model = model
        self.lora = OracleLoRA.init(cfg)
        self.params = self.lora.params(cfg)
        for p in self.params:
            p.requires_grad_(True)
        self.opt = torch.optim.AdamW(
            self.params, lr=cfg.ttt_lora_lr, betas=(cfg.ttt_beta1, cfg.ttt_beta2),
            weight_decay=cfg.ttt_weight_decay,
        )

    def update(self, arr: np.ndarray, end: int) -> float:
        """The lora branch of online_retrain at boundary ``end``
        (compress.py:923-1146): ``_online_steps_at`` steps, the first on the
        newest window, later ones on replay windows (``_replay_window_end``)."""
        from oracle.replenish import online_steps_at, replay_window_end

        cfg = self.model.cfg
        steps = online_steps_at(end, cfg, max(1, int(cfg.online_retrain_every)))
        xy = window_xy(arr, end, cfg.block_size)
        if steps == 0 or xy is None:
            return float("nan")
        x, y = xy
        replay = bool(cfg.online_retrain_replay) and steps > 1
        loss = None
        for si in range(steps):
            if replay and si > 0:
                xy_k = window_xy(arr, replay_window_end(end, si, cfg.seed, cfg.block_size), cfg.block_size)
                if xy_k is not None:
                    x, y = xy_k
            self.opt.zero_grad(set_to_none=True)
            with torch.enable_grad():
                logits = self.model.window_logits(x, self.lora)
                loss = F.cross_entropy(logits.float(), y, reduction="mean")
                loss.backward()
            torch.nn.utils.clip_grad_norm_(self.params, cfg.grad_clip)
            self.opt.step()
        return float(loss.detach())
