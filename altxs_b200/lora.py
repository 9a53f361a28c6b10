"""Host-side pieces shared by the engine: LoRA layout/init and RoPE tables.

LoRA adapters follow the reference ``TTTLoRA`` (altxs
``src/xsa_ttt/ttt_lora.py:22-105``): every adapted projection has
``A [rank, in]`` drawn ``U(-1/sqrt(in), 1/sqrt(in))`` and ``B [out, rank]``
zero, the delta is ``(x @ A.T @ B.T) * alpha / rank``, and an ``lm_head``
adapter is always present.  The initial ``A`` matrices come from one CPU
generator seeded with ``seed ^ 0xA5A51070`` (compress.py:1965-1968) in the
reference's creation order: lm_head, q (per layer), v, k, mlp, o.  The MLP
adapter maps the MLP's normed input (d -> d) and adds to the MLP output; the
o adapter reads the block's normed input, or the attention output with
``ttt_o_lora_on_y`` (ttt_lora.py:161-175).

RoPE tables use the reference ``Rotary`` rule (model.py:130-190): fp32
``inv_freq = 1 / base ** (arange(0, rd, 2) / rd)``, ``freqs = outer(t,
inv_freq)`` at absolute positions ``t``, then ``cos``/``sin``.
"""

from __future__ import annotations

import math
from collections import OrderedDict

import numpy as np
import torch

from .config import ModelConfig


def lora_shapes(cfg: ModelConfig) -> "OrderedDict[str, tuple[tuple[int, int], tuple[int, int]]]":
    """name -> ((rank, in), (out, rank)) in TTTLoRA.parameters() order; one
    adapter slot per layer application (depth loops repeat layers, each
    application with its own adapters: ttt_lora.py:73-77)."""
    r, d, kv, V, L = cfg.ttt_lora_rank, cfg.model_dim, cfg.kv_dim, cfg.vocab_size, cfg.num_virtual_layers
    out: OrderedDict = OrderedDict()
    if not cfg.lora_enabled:
        return out
    out["lm"] = ((r, d), (V, r))
    for i in range(L):
        out[f"q{i}"] = ((r, d), (d, r))
    for i in range(L):
        out[f"v{i}"] = ((r, d), (kv, r))
    if cfg.ttt_k_lora:
        for i in range(L):
            out[f"k{i}"] = ((r, d), (kv, r))
    if cfg.ttt_mlp_lora:
        for i in range(L):
            out[f"mlp{i}"] = ((r, d), (d, r))
    if cfg.ttt_o_lora:
        for i in range(L):
            out[f"o{i}"] = ((r, d), (d, r))
    return out


def init_lora_A(cfg: ModelConfig) -> "OrderedDict[str, np.ndarray]":
    """Initial A matrices (fp32), bit-identical to the reference init."""
    g = torch.Generator()
    g.manual_seed(int(cfg.seed) ^ 0xA5A51070)
    out: OrderedDict = OrderedDict()
    for name, (a_shape, _b_shape) in lora_shapes(cfg).items():
        bound = 1.0 / math.sqrt(a_shape[1])
        a = torch.empty(a_shape).uniform_(-bound, bound, generator=g)
        out[name] = a.numpy().astype(np.float32)
    return out


def rope_tables(cfg: ModelConfig, n_pos: int) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin ``[n_pos, rope_dims/2]`` fp32 at absolute positions."""
    rd = cfg.rope_dims
    inv_freq = 1.0 / cfg.rope_base ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd)
    t = torch.arange(n_pos, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return freqs.cos().numpy().copy(), freqs.sin().numpy().copy()
