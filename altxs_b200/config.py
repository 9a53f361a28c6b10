"""Model and run configuration for the B200 model-and-code loop.

``ModelConfig`` mirrors the subset of the reference ``XsaTttConfig``
(altxs ``src/xsa_ttt/config.py:20-189``) that the per-symbol loop reads.  The
reference motifs that sit on top of the plain GPT (XSA, SmearGate,
SparseAttnGate, depth loops, parallel residual lanes, asymmetric softcap) run
in the decode step and in the full-parameter updates; ``from_reference_cfg`` refuses the
ones this engine does not compute (output gates, YaRN, untied heads) instead
of silently computing a different model.

The always-on pieces of the reference block are kept: QK-RMSNorm, per-head
``q_gain``, partial RoPE over ``rope_dims``, ``resid_mix`` against ``x0``,
``attn_scale``/``mlp_scale``, ``ln_scale = 1/sqrt(layer+1)``,
LeakyReLU(0.5)^2 MLP, tied embeddings with ``softcap * tanh(logits/softcap)``,
U-Net skips with sigmoid skip gates (altxs ``src/xsa_ttt/model.py:885-979,
1377-1476``).
"""

from __future__ import annotations

import dataclasses
import hashlib
import json
from dataclasses import dataclass, field
from typing import Any


@dataclass
class ModelConfig:
    vocab_size: int = 16384
    num_layers: int = 8
    model_dim: int = 512
    num_heads: int = 8
    num_kv_heads: int = 8
    mlp_mult: float = 4.0
    rope_base: float = 1e4
    rope_dims: int = 16
    qk_gain_init: float = 5.0
    logit_softcap: float = 30.0
    ln_scale: bool = True
    skip_gates_enabled: bool = True
    tied_embed_init_std: float = 0.005
    # sequence / lockstep (reference: block_size / online_retrain_every)
    block_size: int = 2048
    online_retrain_every: int = 16384
    # context across segments: "sliding" keeps the last block_size tokens in a
    # ring at absolute positions (this engine's default); "reset" rebuilds the
    # context from the previous block_size symbols at positions 0.. after every
    # boundary update and attends to the whole segment (the reference engine's
    # reset_segment, incremental.py:858-897)
    context_mode: str = "sliding"
    seed: int = 1337
    # test-time LoRA (reference ttt_* fields, config.py:144-165)
    retrain_mode: str = "lora"  # "lora", "replenish" / "full" (every parameter, see below) or "none"
    ttt_lora_rank: int = 8
    ttt_lora_alpha: float = 144.0
    ttt_lora_lr: float = 1e-3
    ttt_beta1: float = 0.0
    ttt_beta2: float = 0.99
    ttt_weight_decay: float = 0.0
    ttt_k_lora: bool = True
    ttt_o_lora: bool = True
    ttt_mlp_lora: bool = False   # MLP adapter (d -> d on the MLP's normed input); reference default on
    ttt_o_lora_on_y: bool = False  # the o adapter reads the attention output instead of the normed input
    ttt_use_rslora: bool = False
    grad_clip: float = 1.0
    # full-parameter replenish (reference config.py:59-138, compress.py:363-482,
    # 611-720, 816-1146): AdamW over every weight of the model on the chunk just
    # coded (with the preceding block as context), optionally Forward-XM over
    # update scales scored on held-out probe chunks
    online_retrain_steps: int = 1
    online_retrain_replay: bool = True
    ttt_bootstrap_symbols: int = 0
    ttt_bootstrap_steps: int = 0
    ttt_replenish_ramp: int = 0
    ttt_replenish_anneal: str = "exp"
    ttt_replenish_lr_half_mb: float = 0.0
    ttt_replenish_lr_min: float = 4e-5
    ttt_replenish_steps_min: int = 1
    ttt_replenish_warmup_steps: int = 16
    ttt_replenish_total_bytes: int = 0
    ttt_replenish_accum: bool = False
    ttt_replenish_replay_lr_scale: float = 1.0
    ttt_replenish_replay_recent_mb: float = 1.0
    ttt_replenish_anchor: str = ""         # safetensors of per-weight stiffness masks ("" = none)
    ttt_replenish_anchor_rate: float = 0.05
    ttt_replenish_xm_k: int = 3
    ttt_replenish_xm_probe_chunks: int = 1
    ttt_replenish_xm_4x_until_bytes: int = 100 * 1024 * 1024
    ttt_burst_schedule: str = ""           # "pos:steps,..." extra steps at the first boundary >= pos
    # "full" mode (the reference's default, compress.py:923-1146): the window loss
    # of the last block_size symbols, replay windows, and burst steps on their own
    # AdamW that walk the segment boundaries oldest -> newest
    ttt_burst_lr: float = 3e-4
    ttt_burst_beta1: float = 0.9
    ttt_burst_beta2: float = 0.999
    ttt_burst_weight_decay: float = 0.01
    # reference model motifs (model.py:982-1110; all off = the plain GPT).  The
    # step, the oracle, every test-time update (lora, replenish, full) and the
    # segment-reset prefill run them.
    smear_gate_enabled: bool = False      # previous-token smear on the raw embedding
    gate_window: int = 12                 # input width of the smear / attention gates
    xsa_last_n: int = 0                   # XSA (value-direction removal) on the last n layers
    sparse_attn_gate_enabled: bool = False  # per-head sigmoid gate on the attention output
    sparse_attn_gate_scale: float = 0.5
    sparse_attn_gate_init_std: float = 0.0  # init draw of the gate weights (Init(seed) of residual codecs)
    asym_logit_rescale: bool = False      # learned positive / negative softcaps
    num_loops: int = 0                    # depth recurrence over layers loop_start..loop_end
    loop_start: int = 3
    loop_end: int = 5
    parallel_start_layer: int = 0         # parallel attention / MLP lanes from this layer (0 = off)
    parallel_final_lane: str = "mean"     # "mean" | "attn" | "mlp"
    # framework CDF rule: "fixed" (integer fixed-point softmax, total
    # <= 2^cdf_bits) or "ref" (reference max(1, floor(p*1e6+0.5)) masses)
    cdf_mode: str = "fixed"
    cdf_bits: int = 20

    # ---- derived ---------------------------------------------------------
    @property
    def head_dim(self) -> int:
        return self.model_dim // self.num_heads

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def mlp_hidden(self) -> int:
        return int(self.mlp_mult * self.model_dim)

    @property
    def layer_schedule(self) -> tuple[list[int], list[int]]:
        """Physical layer of every encoder and decoder application (model.py:1065-1077):
        with depth loops the segment loop_start..loop_end runs num_loops+1 times."""
        L = self.num_layers
        if self.num_loops > 0:
            seg = list(range(self.loop_start, self.loop_end + 1))
            order = list(range(self.loop_start)) + seg * (self.num_loops + 1) + list(range(self.loop_end + 1, L))
            n_enc = len(order) // 2
            return order[:n_enc], order[n_enc:]
        return list(range(L // 2)), list(range(L // 2, L))

    @property
    def num_virtual_layers(self) -> int:
        enc, dec = self.layer_schedule
        return len(enc) + len(dec)

    @property
    def num_encoder_layers(self) -> int:
        return len(self.layer_schedule[0])

    @property
    def num_skip_weights(self) -> int:
        enc, dec = self.layer_schedule
        return min(len(enc), len(dec))

    @property
    def motifs(self) -> bool:
        return bool(self.smear_gate_enabled or self.xsa_last_n > 0 or self.sparse_attn_gate_enabled
                    or self.asym_logit_rescale or self.num_loops > 0 or self.parallel_start_layer > 0)

    @property
    def ctx(self) -> int:
        return self.block_size

    @property
    def kv_len(self) -> int:
        """Rows of the per-stream KV ring: the window, or context + segment."""
        if self.context_mode == "reset":
            return self.block_size + self.online_retrain_every
        return self.block_size

    @property
    def lora_scale(self) -> float:
        r = float(self.ttt_lora_rank)
        if self.ttt_use_rslora:
            return float(self.ttt_lora_alpha) / r**0.5
        return float(self.ttt_lora_alpha) / r

    @property
    def lora_enabled(self) -> bool:
        return self.retrain_mode == "lora" and self.ttt_lora_rank > 0

    def validate(self) -> None:
        if self.model_dim % self.num_heads:
            raise ValueError("model_dim must be divisible by num_heads")
        if self.num_heads % self.num_kv_heads:
            raise ValueError("num_heads must be divisible by num_kv_heads")
        if self.head_dim % 2 or self.rope_dims % 2 or self.rope_dims > self.head_dim:
            raise ValueError("head_dim and rope_dims must be even, rope_dims <= head_dim")
        for k in (self.model_dim, self.mlp_hidden):
            if k % 64:
                raise ValueError("model_dim and mlp hidden must be multiples of 64")
        if self.head_dim > 128 or self.head_dim % 8:
            raise ValueError("head_dim must be a multiple of 8 and <= 128")
        if self.vocab_size < 2:
            raise ValueError("vocab_size must be >= 2")
        if self.cdf_mode not in ("fixed", "ref"):
            raise ValueError("cdf_mode must be 'fixed' or 'ref'")
        if self.cdf_mode == "fixed" and not (self.vocab_size < (1 << self.cdf_bits) <= (1 << 30)):
            raise ValueError("cdf_bits must satisfy vocab < 2^cdf_bits <= 2^30")
        if self.lora_enabled and not 1 <= self.ttt_lora_rank <= 128:
            raise ValueError("ttt_lora_rank must be in 1..128")
        if self.retrain_mode not in ("lora", "replenish", "full", "none"):
            raise ValueError("retrain_mode must be 'lora', 'replenish', 'full' or 'none'")
        if self.retrain_mode in ("replenish", "full") and self.parallel_start_layer > 0:
            dec = self.layer_schedule[1]
            par = [i >= self.parallel_start_layer for i in dec]
            if any(p and not q for p, q in zip(par, par[1:])):
                raise ValueError("the full-parameter update needs every decoder application after the first "
                                 "parallel one to run parallel lanes")
        if self.context_mode not in ("sliding", "reset"):
            raise ValueError("context_mode must be 'sliding' or 'reset'")
        if self.parallel_final_lane not in ("mean", "attn", "mlp"):
            raise ValueError("parallel_final_lane must be 'mean', 'attn' or 'mlp'")
        if self.num_loops > 0 and not (0 <= self.loop_start <= self.loop_end < self.num_layers):
            raise ValueError("loop_start..loop_end must be layers of the model")
        if (self.smear_gate_enabled or self.sparse_attn_gate_enabled) and not 0 < self.gate_window <= self.model_dim:
            raise ValueError("gate_window must be in 1..model_dim")
        if self.sparse_attn_gate_enabled and self.gate_window > self.head_dim:
            raise ValueError("the sparse attention gate needs gate_window <= head_dim")

    def to_dict(self) -> dict[str, Any]:
        return dataclasses.asdict(self)

    def fingerprint(self) -> str:
        """Hash of every field that changes the bitstream (lockstep key)."""
        blob = json.dumps(self.to_dict(), sort_keys=True).encode()
        return hashlib.sha256(blob).hexdigest()[:16]

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "ModelConfig":
        names = {f.name for f in dataclasses.fields(cls)}
        return cls(**{k: v for k, v in d.items() if k in names})

    @classmethod
    def from_reference_cfg(cls, ref: Any) -> "ModelConfig":
        """Map a reference ``XsaTttConfig`` (object or dict) onto this engine."""
        get = (lambda k, dflt=None: ref.get(k, dflt)) if isinstance(ref, dict) else (
            lambda k, dflt=None: getattr(ref, k, dflt)
        )
        unsupported = {
            "attn_out_gate_enabled": bool(get("attn_out_gate_enabled", False)),
            "gated_attn_enabled": bool(get("gated_attn_enabled", False)),
            "rope_yarn": bool(get("rope_yarn", False)),
            "tie_embeddings": not bool(get("tie_embeddings", True)),
        }
        bad = [k for k, v in unsupported.items() if v]
        if bad:
            raise ValueError(f"reference motifs not supported by this engine: {bad}")
        out = cls()
        for f in dataclasses.fields(cls):
            v = get(f.name, None)
            if v is not None:
                setattr(out, f.name, v)
        if out.retrain_mode not in ("lora", "replenish", "full", "none"):
            out.retrain_mode = "none"
        return out


def c1_config() -> ModelConfig:
    """CPU plumbing config: 2L/128d/4h, ctx 256, V 4096, rank-4 q/v LoRA
    (plus the lm_head adapter) updated every 4096 symbols at lr 1e-3, 16-bit
    CDF precision.  Its weights are the reference's seed-0 init
    (``codec.reference_init(cfg, 0)``)."""
    return ModelConfig(
        vocab_size=4096, num_layers=2, model_dim=128, num_heads=4, num_kv_heads=4,
        mlp_mult=4.0, block_size=256, online_retrain_every=4096, seed=0,
        ttt_lora_rank=4, ttt_lora_lr=1e-3, ttt_k_lora=False, ttt_o_lora=False, cdf_bits=16,
    )


def c3_config() -> ModelConfig:
    """33M config: 8L/512d/8h (hd 64, MHA), MLP 2048, V 16384, ctx 2048."""
    return ModelConfig(
        vocab_size=16384, num_layers=8, model_dim=512, num_heads=8, num_kv_heads=8,
        mlp_mult=4.0, block_size=2048, online_retrain_every=16384, seed=1337,
        ttt_lora_rank=8, ttt_lora_lr=1e-3, ttt_k_lora=True, ttt_o_lora=True,
    )


@dataclass
class RunStats:
    """Per-run counters reported by the entry points."""

    n_symbols: int = 0
    payload_bytes: int = 0
    retrain_count: int = 0
    segments: list = field(default_factory=list)
