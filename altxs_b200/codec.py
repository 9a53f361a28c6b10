"""Mixed-bit weight format: the reference v5 codec on disk, a group layout on device.

On disk this reads and writes the reference's ``hope_mixed_bit_delta`` v5
format (altxs ``src/hyperflow_distillation/mixed_bit_delta.py``): a
safetensors file with ``bits/<bank>``, ``packed/<bank>/b{2,3,4}``,
``codebook/<bank>/b{b}`` and ``small/<param>`` tensors plus a sibling JSON
with ``layouts``/``codebook_mode``/``cfg``/``small_params``.  Codes are
packed LSB-first with 3-bit codes as 8 per 3 bytes (``unpack_codes``,
mixed_bit_delta.py:96-113); channels of one bit width are concatenated in
channel order; ``symmetric`` codebooks hold one fp16 scale per channel with
levels ``(i - (2^b-1)/2) * s`` (:147-152, :209-213) and ``lloyd`` codebooks
hold 2^b fp16 centroids per channel (:203-208).

Channel orientation.  The reference splits each bank into channels of
``channel_width`` values: rows of q/k/v/up/emb, and *columns* of o and
mlp_down (stored transposed, ``_from_channels`` :116-144).  The benchmark
configs instead quantise every matrix in 64-wide groups along the input
dimension K; such codecs carry ``"channel_axis": "in"`` in the JSON and
every bank is chunked row-major along its input dimension.  Reference-layout
codecs are also read: transposed channels cannot share one codebook per
K-group, so those matrices become dense fp32 groups (exact values).

``"delta_base": "zero"`` marks codecs whose dequantised values ARE the
weights (the synthetic benchmark model).  Reference codecs are residuals on
``Init(seed)`` (mixed_bit_delta.py:232-305); that base is not rebuilt here.

On device every matrix ``W[rows, cols]`` is a ``PackedMatrix``: per row,
groups of 64 along ``cols`` with a 32-bit descriptor each
``[scale fp16 | width code << 16 | in-row offset (8-byte units) << 20]``,
the group's codes packed LSB-first in ``8*bits`` bytes (256 bytes of raw
fp32 for dense groups), and ``row_off8[rows]`` giving each row's first byte
in 8-byte units.  The kernels compute, for every output,
``y = sum_g fma(scale_g, sum_i fma(level_i, x_i), y)`` in a fixed order.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np

from .config import ModelConfig
from .synth import GROUP, synth_groups

FORMAT = "hope_mixed_bit_delta"
FORMAT_VERSION = 5
WIDTH_CODE = {0: 0, 2: 1, 3: 2, 4: 3, 32: 4}
BANKS = ("qo_bank", "kv_bank", "mlp_up_bank", "mlp_down_bank", "tok_emb.weight")


# ---------------------------------------------------------------------------
# group matrices (host form)
# ---------------------------------------------------------------------------


@dataclass
class GroupMatrix:
    """``[rows, cols]`` weights as 64-wide groups along ``cols``.

    ``bits`` in {0, 2, 3, 4, 32}; ``codes`` holds the quantised codes
    (ignored for 0/32-bit groups); ``scales`` the fp16 group scale (1.0 for
    codebook groups); ``lut``/``glut`` give optional per-group codebooks
    (lloyd mode); ``dense`` the fp32 values of 32-bit groups.
    """

    bits: np.ndarray  # [rows, G] uint8
    codes: np.ndarray  # [rows, cols] uint8
    scales: np.ndarray  # [rows, G] float16
    lut: np.ndarray | None = None  # [n_lut, 16] float16
    glut: np.ndarray | None = None  # [rows, G] uint32
    dense: np.ndarray | None = None  # [rows, cols] float32

    @property
    def shape(self) -> tuple[int, int]:
        return int(self.codes.shape[0]), int(self.codes.shape[1])

    def dequant(self) -> np.ndarray:
        rows, cols = self.shape
        b = np.repeat(self.bits, GROUP, axis=1)
        code = self.codes.astype(np.int64)
        if self.lut is not None:
            li = np.repeat(self.glut.astype(np.int64), GROUP, axis=1)
            lev = self.lut.astype(np.float32)[li, code]
        else:
            center = (np.float32(2.0) ** b.astype(np.float32) - np.float32(1.0)) / np.float32(2.0)
            lev = code.astype(np.float32) - center
        out = lev * np.repeat(self.scales.astype(np.float32), GROUP, axis=1)
        out = out.astype(np.float32)
        out[b == 0] = 0.0
        if self.dense is not None:
            m = b == 32
            out[m] = self.dense[m]
        return out

    @classmethod
    def from_dense(cls, w: np.ndarray) -> "GroupMatrix":
        w = np.ascontiguousarray(w, dtype=np.float32)
        rows, cols = w.shape
        if cols % GROUP:
            raise ValueError("cols must be a multiple of 64")
        g = cols // GROUP
        return cls(
            bits=np.full((rows, g), 32, dtype=np.uint8),
            codes=np.zeros((rows, cols), dtype=np.uint8),
            scales=np.ones((rows, g), dtype=np.float16),
            dense=w,
        )

    @classmethod
    def vstack(cls, mats: list["GroupMatrix"]) -> "GroupMatrix":
        luts = [m.lut for m in mats]
        has_lut = any(x is not None for x in luts)
        has_dense = any(m.dense is not None for m in mats)
        lut = glut = dense = None
        if has_lut:
            parts, gparts, base = [], [], 0
            for m in mats:
                if m.lut is None:
                    raise ValueError("cannot stack codebook and symmetric matrices")
                parts.append(m.lut)
                gparts.append(m.glut.astype(np.int64) + base)
                base += m.lut.shape[0]
            lut = np.concatenate(parts)
            glut = np.concatenate(gparts).astype(np.uint32)
        if has_dense:
            dense = np.concatenate(
                [m.dense if m.dense is not None else np.zeros(m.shape, np.float32) for m in mats]
            )
        return cls(
            bits=np.concatenate([m.bits for m in mats]),
            codes=np.concatenate([m.codes for m in mats]),
            scales=np.concatenate([m.scales for m in mats]),
            lut=lut, glut=glut, dense=dense,
        )


@dataclass
class PackedMatrix:
    """Device layout of a ``GroupMatrix`` (numpy arrays, uploaded by the engine)."""

    rows: int
    cols: int
    codes: np.ndarray  # uint8, length multiple of 16
    row_off8: np.ndarray  # uint32 [rows]
    gdesc: np.ndarray  # uint32 [rows, G]
    lut: np.ndarray | None  # float16 [n_lut, 16]
    glut: np.ndarray | None  # uint32 [rows, G]

    @property
    def nbytes(self) -> int:
        n = self.codes.nbytes + self.row_off8.nbytes + self.gdesc.nbytes
        if self.lut is not None:
            n += self.lut.nbytes + self.glut.nbytes
        return n


def _pack_lsb(codes: np.ndarray, bits: int) -> np.ndarray:
    """Pack ``[n, 64]`` codes LSB-first into ``[n, 8*bits]`` bytes."""
    n = codes.shape[0]
    shifts = np.arange(bits, dtype=np.uint8)
    bitarr = ((codes[:, :, None] >> shifts[None, None, :]) & 1).astype(np.uint8)
    return np.packbits(bitarr.reshape(n, GROUP * bits), axis=1, bitorder="little")


def unpack_lsb(packed: np.ndarray, bits: int, count: int) -> np.ndarray:
    """Inverse of the LSB-first packing (any width 1..8)."""
    p = np.asarray(packed, dtype=np.uint8).reshape(-1)
    bitarr = np.unpackbits(p, bitorder="little")[: count * bits].reshape(count, bits)
    weights = (1 << np.arange(bits)).astype(np.uint16)
    return (bitarr.astype(np.uint16) * weights[None, :]).sum(axis=1).astype(np.uint8)


def pack_matrix(m: GroupMatrix) -> PackedMatrix:
    rows, cols = m.shape
    g = cols // GROUP
    bits = m.bits.astype(np.int64)
    bad = ~np.isin(bits, list(WIDTH_CODE))
    if bad.any():
        raise ValueError(f"unsupported group widths {np.unique(bits[bad])}")
    units = bits  # 8-byte units per group: 64*b bits = 8*b bytes
    goff = np.zeros_like(units)
    goff[:, 1:] = np.cumsum(units, axis=1)[:, :-1]
    if goff.size and goff.max() >= 4096:
        raise ValueError("row too wide for the 12-bit in-row offset")
    row_units = units.sum(axis=1)
    row_off8 = np.zeros(rows, dtype=np.int64)
    row_off8[1:] = np.cumsum(row_units)[:-1]
    total_units = int(row_units.sum())
    if total_units >= (1 << 32):
        raise ValueError("matrix too large for 32-bit row offsets")
    nbytes = total_units * 8
    codes_out = np.zeros(max(16, (nbytes + 15) // 16 * 16), dtype=np.uint8)
    byte_base = (row_off8[:, None] + goff) * 8  # [rows, G]
    codes_g = m.codes.reshape(rows, g, GROUP)
    for b in (2, 3, 4):
        r_idx, g_idx = np.nonzero(bits == b)
        if r_idx.size == 0:
            continue
        packed = _pack_lsb(codes_g[r_idx, g_idx], b)  # [n, 8b]
        dst = byte_base[r_idx, g_idx][:, None] + np.arange(8 * b)[None, :]
        codes_out[dst] = packed
    r_idx, g_idx = np.nonzero(bits == 32)
    if r_idx.size:
        vals = m.dense.reshape(rows, g, GROUP)[r_idx, g_idx].astype("<f4")
        raw = vals.view(np.uint8).reshape(r_idx.size, 256)
        dst = byte_base[r_idx, g_idx][:, None] + np.arange(256)[None, :]
        codes_out[dst] = raw
    wcode = np.vectorize(WIDTH_CODE.get, otypes=[np.int64])(bits) if bits.size else bits
    scale_bits = m.scales.astype(np.float16).view(np.uint16).astype(np.int64)
    gdesc = (scale_bits | (wcode << 16) | (goff << 20)).astype(np.uint32)
    return PackedMatrix(
        rows=rows, cols=cols, codes=codes_out,
        row_off8=row_off8.astype(np.uint32), gdesc=gdesc.reshape(rows, g),
        lut=None if m.lut is None else np.ascontiguousarray(m.lut, dtype=np.float16),
        glut=None if m.glut is None else np.ascontiguousarray(m.glut, dtype=np.uint32),
    )


TILE_ROWS = 64
TILE_SEG = 256 + TILE_ROWS * 32  # 64 group descriptors, then up to 64 groups of <= 32 code bytes


def tile_stream(p: PackedMatrix) -> np.ndarray | None:
    """The packed codes re-laid for the tensor-core GEMM's producer: one
    fixed-size segment of TILE_SEG bytes per (64-row block, 64-wide group),
    ``[ceil(rows/64)][cols/64][TILE_SEG]`` uint8, so that a tile's K slice is
    one bulk copy with no table lookups.  Segment = 64 uint32 descriptors
    (fp16 scale | width code << 16 | offset of the row's code bytes within the
    segment's code area, 8-byte units, << 20) followed by the rows' code
    bytes (8*b each, as in the packed rows).  Rows past the matrix are 0-bit
    groups.  None when a group is not 0/2/3/4-bit symmetric (codebook or
    exact fp32 groups): such matrices keep the dense planes."""
    if p.lut is not None:
        return None
    rows, cols = p.rows, p.cols
    G = cols // GROUP
    wcode = ((p.gdesc >> 16) & 15).astype(np.int64)
    if np.any(wcode > 3):
        return None
    size = np.array([0, 16, 24, 32], dtype=np.int64)[wcode]  # [rows, G] bytes
    RB = (rows + TILE_ROWS - 1) // TILE_ROWS
    pad = RB * TILE_ROWS - rows
    size_p = np.pad(size, ((0, pad), (0, 0)))
    desc_p = np.pad(p.gdesc.astype(np.int64), ((0, pad), (0, 0)))
    # [RB, 64, G] -> offsets of each row's bytes within its (block, group) segment
    sz = size_p.reshape(RB, TILE_ROWS, G)
    off = np.cumsum(sz, axis=1) - sz  # exclusive, bytes
    tdesc = (desc_p.reshape(RB, TILE_ROWS, G) & 0xFFFF) | (np.pad(wcode, ((0, pad), (0, 0))).reshape(
        RB, TILE_ROWS, G) << 16) | ((off // 8) << 20)
    out = np.zeros((RB, G, TILE_SEG), dtype=np.uint8)
    out[:, :, :256] = np.ascontiguousarray(tdesc.transpose(0, 2, 1)).astype("<u4").view(np.uint8).reshape(RB, G, 256)
    # code bytes: source [row_off8 + goff] * 8 in the packed rows
    r_idx, g_idx = np.nonzero(size > 0)
    if r_idx.size:
        n = size[r_idx, g_idx]
        src0 = (p.row_off8[r_idx].astype(np.int64) + (p.gdesc[r_idx, g_idx].astype(np.int64) >> 20)) * 8
        dst0 = ((r_idx // TILE_ROWS) * G + g_idx) * TILE_SEG + 256 + off.reshape(RB * TILE_ROWS, G)[r_idx, g_idx]
        rep = np.repeat(np.arange(r_idx.size), n)
        within = np.arange(rep.size) - np.repeat(np.cumsum(n) - n, n)
        out.reshape(-1)[dst0[rep] + within] = p.codes[src0[rep] + within]
    return out


# ---------------------------------------------------------------------------
# model weights
# ---------------------------------------------------------------------------


@dataclass
class ModelWeights:
    """All weights of one model in group form plus the small fp32 params."""

    cfg: ModelConfig
    emb: GroupMatrix  # [V, d]
    q: list[GroupMatrix]  # [d, d]
    k: list[GroupMatrix]  # [kv, d]
    v: list[GroupMatrix]  # [kv, d]
    o: list[GroupMatrix]  # [d, d]
    up: list[GroupMatrix]  # [F, d]
    down: list[GroupMatrix]  # [d, F]
    small: dict[str, np.ndarray]

    def dense(self) -> dict[str, Any]:
        """Dense fp32 tensors in the reference's parameter naming."""
        cfg = self.cfg
        L = cfg.num_layers
        out: dict[str, Any] = {
            "tok_emb.weight": self.emb.dequant(),
            "qo_bank": np.stack([m.dequant() for m in self.q] + [m.dequant() for m in self.o]),
            "kv_bank": np.stack([m.dequant() for m in self.k] + [m.dequant() for m in self.v]),
            "mlp_up_bank": np.stack([m.dequant() for m in self.up]),
            "mlp_down_bank": np.stack([m.dequant() for m in self.down]),
        }
        assert out["qo_bank"].shape[0] == 2 * L
        out.update(self.small_reference_names())
        return out

    def small_reference_names(self) -> dict[str, np.ndarray]:
        s = self.small
        out = {
            "skip_weights": s["skip_weights"],
            "skip_gates": s["skip_gates"],
        }
        for i in range(self.cfg.num_layers):
            out[f"blocks.{i}.attn_scale"] = s["attn_scale"][i]
            out[f"blocks.{i}.mlp_scale"] = s["mlp_scale"][i]
            out[f"blocks.{i}.resid_mix"] = s["resid_mix"][i]
            out[f"blocks.{i}.attn.q_gain"] = s["q_gain"][i]
        return out

    def packed(self) -> dict[str, PackedMatrix]:
        """Device layout: emb, and per-layer-stacked qkv / o / up / down."""
        L = self.cfg.num_layers
        qkv = GroupMatrix.vstack(
            [GroupMatrix.vstack([self.q[i], self.k[i], self.v[i]]) for i in range(L)]
        )
        return {
            "emb": pack_matrix(self.emb),
            "qkv": pack_matrix(qkv),
            "o": pack_matrix(GroupMatrix.vstack(self.o)),
            "up": pack_matrix(GroupMatrix.vstack(self.up)),
            "down": pack_matrix(GroupMatrix.vstack(self.down)),
        }

    @property
    def bits_per_weight(self) -> float:
        mats = [self.emb, *self.q, *self.k, *self.v, *self.o, *self.up, *self.down]
        tot = sum(float(m.bits.astype(np.float64).sum()) * GROUP for m in mats)
        n = sum(m.codes.size for m in mats)
        return tot / n


def default_small(cfg: ModelConfig) -> dict[str, np.ndarray]:
    """Reference init of the small parameters (model.py:925-930, 1081-1090)."""
    L, d, H, S = cfg.num_layers, cfg.model_dim, cfg.num_heads, cfg.num_skip_weights
    rm = np.zeros((L, 2, d), dtype=np.float32)
    rm[:, 0, :] = 1.0
    gw = cfg.gate_window
    return {
        "q_gain": np.full((L, H), cfg.qk_gain_init, dtype=np.float32),
        "attn_scale": np.ones((L, d), dtype=np.float32),
        "mlp_scale": np.ones((L, d), dtype=np.float32),
        "resid_mix": rm,
        "skip_weights": np.ones((S, d), dtype=np.float32),
        "skip_gates": np.zeros((S, d), dtype=np.float32),
        # motifs (model.py:994-996, 1087-1105, 753-758): zero-initialised gates, unit lambdas
        "smear_gate": np.zeros((gw,), dtype=np.float32),
        "smear_lambda": np.zeros((1,), dtype=np.float32),
        "attn_gate_w": np.zeros((L, H, gw), dtype=np.float32),
        "softcap": np.array([cfg.logit_softcap, cfg.logit_softcap], dtype=np.float32),  # positive, negative
        "parallel_post": np.ones((L, 2, 2), dtype=np.float32),
        "parallel_resid": np.full((L, 2), 1.1, dtype=np.float32),
    }


def synth_weights(cfg: ModelConfig, seed: int = 0) -> ModelWeights:
    """Seeded random mixed-bit model (the benchmark's 3.15-bpw weights)."""
    cfg.validate()
    rng = np.random.default_rng(np.random.SeedSequence([int(seed), 0xA17C5]))
    d, kv, F, L = cfg.model_dim, cfg.kv_dim, cfg.mlp_hidden, cfg.num_layers

    def mat(rows: int, cols: int) -> GroupMatrix:
        b, c, s = synth_groups(rows, cols, rng)
        return GroupMatrix(bits=b, codes=c, scales=s)

    emb = mat(cfg.vocab_size, d)
    q = [mat(d, d) for _ in range(L)]
    o = [mat(d, d) for _ in range(L)]
    k = [mat(kv, d) for _ in range(L)]
    v = [mat(kv, d) for _ in range(L)]
    up = [mat(F, d) for _ in range(L)]
    down = [mat(d, F) for _ in range(L)]
    return ModelWeights(cfg, emb, q, k, v, o, up, down, default_small(cfg))


def small_from_state(cfg: ModelConfig, tensors: dict[str, Any]) -> dict[str, np.ndarray]:
    """The engine's small parameters from reference-named tensors; names that
    are absent keep the reference's initial values."""
    L = cfg.num_layers

    def t(name):
        x = tensors[name]
        return np.asarray(x.detach().cpu().numpy() if hasattr(x, "detach") else x, dtype=np.float32)

    small = default_small(cfg)
    for name in ("skip_weights", "skip_gates"):
        if name in tensors and np.size(tensors[name]):
            small[name] = t(name).reshape(-1, cfg.model_dim)
    for i in range(L):
        for field, key in (("attn_scale", "attn_scale"), ("mlp_scale", "mlp_scale"), ("resid_mix", "resid_mix"),
                           ("q_gain", "attn.q_gain"), ("attn_gate_w", "attn.attn_gate_w")):
            name = f"blocks.{i}.{key}"
            if name in tensors:
                small[field][i] = t(name).reshape(small[field][i].shape)
    if "smear_gate.weight" in tensors:
        small["smear_gate"] = t("smear_gate.weight").reshape(-1)
    if "smear_lambda" in tensors:
        small["smear_lambda"] = t("smear_lambda").reshape(1)
    if "softcap_pos" in tensors:
        small["softcap"] = np.array([float(t("softcap_pos")), float(t("softcap_neg"))], dtype=np.float32)
    if "parallel_post_lambdas" in tensors:
        small["parallel_post"] = t("parallel_post_lambdas").reshape(L, 2, 2)
    if "parallel_resid_lambdas" in tensors:
        small["parallel_resid"] = t("parallel_resid_lambdas").reshape(L, 2)
    return small


def reference_init(cfg: ModelConfig, seed: int) -> dict[str, np.ndarray]:
    """The reference's deterministic ``Init(seed)`` (``build_model`` after
    ``enable_deterministic``: ``torch.manual_seed(seed)``, then ``GPT.__init__``
    and ``_init_weights``, altxs src/xsa_ttt/model.py:985-1163,
    src/model/deterministic_mode.py:50-62), as reference-named fp32 arrays.

    The draws from torch's CPU generator are replayed in construction order:
    ``nn.Embedding`` N(0,1); per block the sparse attention gate
    N(0, init_std) when that std is positive; the smear gate's ``nn.Linear``
    Kaiming-uniform draw (then zeroed); in ``_init_weights`` the tied table
    N(0, tied_embed_init_std), per layer orthogonal q, k, v (o zero), then per
    layer orthogonal up (down zero).  ``orthogonal_`` is torch's QR recipe with
    the same generator, so the values are torch's own."""
    import math as _m

    import torch

    V, L, d, H, kv, F = (cfg.vocab_size, cfg.num_layers, cfg.model_dim, cfg.num_heads, cfg.kv_dim,
                         cfg.mlp_hidden)
    g = torch.Generator().manual_seed(int(seed))

    def orthogonal(rows: int, cols: int) -> torch.Tensor:
        flat = torch.empty(rows, cols).normal_(0.0, 1.0, generator=g)
        if rows < cols:
            flat = flat.t()
        q, r = torch.linalg.qr(flat)
        q = q * torch.diag(r, 0).sign()
        if rows < cols:
            q = q.t()
        return q.contiguous()

    emb = torch.empty(V, d).normal_(0.0, 1.0, generator=g)
    gate_w = torch.zeros(L, H, cfg.gate_window)
    for i in range(L):
        if cfg.sparse_attn_gate_enabled and cfg.sparse_attn_gate_init_std > 0:
            gate_w[i] = torch.empty(H, cfg.gate_window).normal_(0.0, float(cfg.sparse_attn_gate_init_std),
                                                                 generator=g)
    if cfg.smear_gate_enabled:  # nn.Linear(gate_window, 1).reset_parameters, later zero-initialised
        bound = 1.0 / _m.sqrt(cfg.gate_window)
        torch.empty(1, cfg.gate_window).uniform_(-bound, bound, generator=g)
    emb.normal_(0.0, float(cfg.tied_embed_init_std), generator=g)
    qo = torch.zeros(2 * L, d, d)
    kvb = torch.zeros(2 * L, kv, d)
    up = torch.zeros(L, F, d)
    for i in range(L):
        qo[i] = orthogonal(d, d)
        kvb[i] = orthogonal(kv, d)
        kvb[L + i] = orthogonal(kv, d)
    for i in range(L):
        up[i] = orthogonal(F, d)
    out = {"tok_emb.weight": emb, "qo_bank": qo, "kv_bank": kvb, "mlp_up_bank": up,
           "mlp_down_bank": torch.zeros(L, d, F)}
    small = default_small(cfg)
    S = cfg.num_skip_weights
    out["skip_weights"] = torch.ones(S, d)
    if cfg.skip_gates_enabled:
        out["skip_gates"] = torch.zeros(S, d)
    for i in range(L):
        out[f"blocks.{i}.attn_scale"] = torch.from_numpy(small["attn_scale"][i])
        out[f"blocks.{i}.mlp_scale"] = torch.from_numpy(small["mlp_scale"][i])
        out[f"blocks.{i}.resid_mix"] = torch.from_numpy(small["resid_mix"][i])
        out[f"blocks.{i}.attn.q_gain"] = torch.from_numpy(small["q_gain"][i])
        if cfg.sparse_attn_gate_enabled:
            out[f"blocks.{i}.attn.attn_gate_w"] = gate_w[i]
    if cfg.smear_gate_enabled:
        out["smear_gate.weight"] = torch.zeros(1, cfg.gate_window)
        out["smear_lambda"] = torch.zeros(1)
    if cfg.asym_logit_rescale:
        out["softcap_pos"] = torch.tensor(float(cfg.logit_softcap))
        out["softcap_neg"] = torch.tensor(float(cfg.logit_softcap))
    out["parallel_post_lambdas"] = torch.ones(L, 2, 2)
    out["parallel_resid_lambdas"] = torch.full((L, 2), 1.1)
    return {k: v.numpy().astype(np.float32) for k, v in out.items()}


def dense_weights(cfg: ModelConfig, tensors: dict[str, Any]) -> ModelWeights:
    """Wrap dense fp32 reference-named tensors (e.g. a reference GPT state
    dict) as 32-bit groups, so the kernels run a dense model exactly."""
    cfg.validate()
    L, d, kv = cfg.num_layers, cfg.model_dim, cfg.kv_dim

    def t(name):
        x = tensors[name]
        return np.asarray(x.detach().cpu().numpy() if hasattr(x, "detach") else x, dtype=np.float32)

    qo, kvb = t("qo_bank"), t("kv_bank")
    up, down = t("mlp_up_bank"), t("mlp_down_bank")
    small = small_from_state(cfg, tensors)
    gm = GroupMatrix.from_dense
    return ModelWeights(
        cfg,
        gm(t("tok_emb.weight")),
        [gm(qo[i]) for i in range(L)],
        [gm(kvb[i]) for i in range(L)],
        [gm(kvb[L + i]) for i in range(L)],
        [gm(qo[L + i]) for i in range(L)],
        [gm(up[i]) for i in range(L)],
        [gm(down[i]) for i in range(L)],
        small,
    )


# ---------------------------------------------------------------------------
# v5 codec files
# ---------------------------------------------------------------------------


def _bank_mats(w: ModelWeights) -> dict[str, list[GroupMatrix]]:
    return {
        "qo_bank": w.q + w.o,
        "kv_bank": w.k + w.v,
        "mlp_up_bank": w.up,
        "mlp_down_bank": w.down,
        "tok_emb.weight": [w.emb],
    }


def _bank_shapes(cfg: ModelConfig) -> dict[str, list[int]]:
    L, d, kv, F, V = cfg.num_layers, cfg.model_dim, cfg.kv_dim, cfg.mlp_hidden, cfg.vocab_size
    return {
        "qo_bank": [2 * L, d, d],
        "kv_bank": [2 * L, kv, d],
        "mlp_up_bank": [L, F, d],
        "mlp_down_bank": [L, d, F],
        "tok_emb.weight": [V, d],
    }


def small_param_tensors(w: ModelWeights) -> dict[str, np.ndarray]:
    return {k: np.asarray(v, dtype=np.float32) for k, v in w.small_reference_names().items()}


def write_codec(w: ModelWeights, path: str | Path) -> Path:
    """Write symmetric group-64 weights as a v5 codec (``channel_axis: in``)."""
    from safetensors.numpy import save_file

    path = Path(path).with_suffix(".safetensors")
    cfg = w.cfg
    tensors: dict[str, np.ndarray] = {}
    layouts: dict[str, Any] = {}
    for name, mats in _bank_mats(w).items():
        if any(m.lut is not None or m.dense is not None for m in mats):
            raise ValueError("write_codec handles symmetric quantised matrices only")
        bits = np.concatenate([m.bits.reshape(-1) for m in mats])
        codes = np.concatenate([m.codes.reshape(-1, GROUP) for m in mats])
        scales = np.concatenate([m.scales.reshape(-1) for m in mats])
        tensors[f"bits/{name}"] = bits.astype(np.uint8)
        counts = {str(b): int((bits == b).sum()) for b in (0, 2, 3, 4)}
        for b in (2, 3, 4):
            idx = np.flatnonzero(bits == b)
            if idx.size:
                tensors[f"packed/{name}/b{b}"] = _pack_lsb(codes[idx], b).reshape(-1)
            else:
                tensors[f"packed/{name}/b{b}"] = np.zeros(0, dtype=np.uint8)
            tensors[f"codebook/{name}/b{b}"] = scales[idx].reshape(-1, 1).astype(np.float16)
        layouts[name] = {
            "shape": _bank_shapes(cfg)[name],
            "channels": int(bits.size),
            "channel_width": GROUP,
            "fp16": False,
            "channel_counts": counts,
        }
    small = small_param_tensors(w)
    for k, v in small.items():
        tensors[f"small/{k}"] = v.astype(np.float16)
    save_file(tensors, str(path))
    meta = {
        "format": FORMAT,
        "format_version": FORMAT_VERSION,
        "seed": int(cfg.seed),
        "cfg": cfg.to_dict(),
        "codebook_mode": "symmetric",
        "channel_axis": "in",
        "delta_base": "zero",
        "n_layers": int(cfg.num_layers),
        "layouts": layouts,
        "small_params": sorted(small),
        "average_bits_per_weight": w.bits_per_weight,
    }
    path.with_suffix(".json").write_text(json.dumps(meta, indent=1) + "\n")
    return path


def _is_transposed(name: str, axis: str, mi: int, n_mats: int) -> bool:
    """Reference layout stores o and mlp_down channels as columns."""
    if axis == "in":
        return False
    if name == "mlp_down_bank":
        return True
    return name == "qo_bank" and mi >= n_mats // 2


def _channels_to_groups(name, bits, codes_of, lut_of, scale_of, width, shape, axis):
    """Map channel arrays onto per-matrix GroupMatrix objects."""
    rows_per = shape[-2] if len(shape) == 3 else shape[0]
    cols = shape[-1]
    n_mats = shape[0] if len(shape) == 3 else 1
    mats = []
    ch = 0
    for mi in range(n_mats):
        if _is_transposed(name, axis, mi, n_mats):
            if width != rows_per:
                raise ValueError(f"{name}: transposed channels must span the output dim")
            sel = np.arange(ch, ch + cols)
            ch += cols
            vals = _dense_from_channels(bits[sel], codes_of(sel), lut_of(sel), scale_of(sel))
            mats.append(GroupMatrix.from_dense(np.ascontiguousarray(vals.T)))
            continue
        if width % GROUP or cols % width:
            raise ValueError(f"{name}: channel_width {width} incompatible with 64-groups")
        g_per_ch = width // GROUP
        n_ch = rows_per * (cols // width)
        sel = np.arange(ch, ch + n_ch)
        ch += n_ch
        gb = np.repeat(bits[sel], g_per_ch).reshape(rows_per, cols // GROUP)
        gcodes = codes_of(sel).reshape(rows_per, cols)
        scales = np.repeat(scale_of(sel), g_per_ch).reshape(rows_per, cols // GROUP)
        lut = glut = None
        lu = lut_of(sel)
        if lu is not None:
            lut, li = lu
            glut = np.repeat(li, g_per_ch).reshape(rows_per, cols // GROUP).astype(np.uint32)
        mats.append(
            GroupMatrix(bits=gb.astype(np.uint8), codes=gcodes,
                        scales=scales.astype(np.float16), lut=lut, glut=glut)
        )
    if ch != bits.size:
        raise ValueError(f"{name}: {bits.size} channels, layout consumed {ch}")
    return mats


def _dense_from_channels(bits, codes, lu, scales):
    """Dense fp32 values of whole channels ``[n_ch, width]``."""
    codes = codes.astype(np.int64)
    if lu is not None:
        lut, li = lu
        vals = lut.astype(np.float32)[li[:, None], codes]
    else:
        center = (np.float32(2.0) ** bits.astype(np.float32) - np.float32(1.0)) / np.float32(2.0)
        vals = (codes.astype(np.float32) - center[:, None]) * scales.astype(np.float32)[:, None]
    vals = vals.astype(np.float32)
    vals[bits == 0] = 0.0
    return vals


def read_codec(path: str | Path) -> ModelWeights:
    """Load a v5 codec into ``ModelWeights`` (symmetric or lloyd codebooks)."""
    from safetensors.numpy import load_file

    path = Path(path).with_suffix(".safetensors")
    meta = json.loads(path.with_suffix(".json").read_text())
    if meta.get("format") != FORMAT:
        raise ValueError(f"not a mixed-bit delta codec: {path}")
    if int(meta.get("format_version", -1)) not in (3, 4, 5):
        raise ValueError(f"unsupported format_version {meta.get('format_version')}")
    residual = meta.get("delta_base", "init") != "zero"
    if meta.get("global_lora"):
        raise ValueError("this codec has a global-LoRA residual; the reference ships no decoder for it")
    if meta.get("compact"):
        raise ValueError("zlib-compacted codecs are not supported")
    mode = str(meta.get("codebook_mode", "lloyd")).lower()
    if mode not in ("symmetric", "lloyd"):
        raise ValueError(f"codebook_mode {mode!r} not supported")
    axis = meta.get("channel_axis", "ref")
    cfg_d = meta.get("cfg") or {}
    # this engine's own configs carry its CDF rule; anything else is a reference XsaTttConfig
    cfg = ModelConfig.from_dict(cfg_d) if "cdf_mode" in cfg_d else ModelConfig.from_reference_cfg(cfg_d)
    cfg.validate()
    st = load_file(str(path))
    L = int(meta["n_layers"])
    banks: dict[str, list[GroupMatrix]] = {}
    for name in BANKS:
        lay = meta["layouts"][name]
        width = int(lay["channel_width"])
        shape = [int(x) for x in lay["shape"]]
        bits = st[f"bits/{name}"].astype(np.uint8)
        codes_by_b, cb_by_b, rank = {}, {}, np.zeros(bits.size, dtype=np.int64)
        for b in (2, 3, 4):
            idx = np.flatnonzero(bits == b)
            rank[idx] = np.arange(idx.size)
            if idx.size:
                codes_by_b[b] = unpack_lsb(st[f"packed/{name}/b{b}"], b, idx.size * width).reshape(idx.size, width)
                cb_by_b[b] = st[f"codebook/{name}/b{b}"]

        def codes_of(sel, bits=bits, codes_by_b=codes_by_b, rank=rank, width=width):
            out = np.zeros((sel.size, width), dtype=np.uint8)
            for b, arr in codes_by_b.items():
                m = bits[sel] == b
                out[m] = arr[rank[sel[m]]]
            return out

        def scale_of(sel, bits=bits, cb_by_b=cb_by_b, rank=rank):
            out = np.ones(sel.size, dtype=np.float16)
            if mode == "symmetric":
                for b, arr in cb_by_b.items():
                    m = bits[sel] == b
                    out[m] = arr.reshape(-1)[rank[sel[m]]]
            return out

        def lut_of(sel, bits=bits, cb_by_b=cb_by_b, rank=rank):
            if mode != "lloyd":
                return None
            lut = np.zeros((sel.size, 16), dtype=np.float16)
            for b, arr in cb_by_b.items():
                m = bits[sel] == b
                lut[m, : 1 << b] = arr[rank[sel[m]]]
            return lut, np.arange(sel.size, dtype=np.int64)

        banks[name] = _channels_to_groups(name, bits, codes_of, lut_of, scale_of, width, shape, axis)
    if residual:
        # the reference's load_codec: Init(seed) + dequantised delta for the banks,
        # the listed small parameters replace their initial values (mixed_bit_delta.py:232-305,
        # train_hyperflow.py:8-19)
        state = reference_init(cfg, int(meta["seed"]))
        for name, mats in banks.items():
            delta = np.concatenate([m.dequant() for m in mats]).reshape(state[name].shape)
            state[name] = (state[name] + delta).astype(np.float32)
        for k in meta["small_params"]:
            if f"small/{k}" in st:
                state[k] = st[f"small/{k}"].astype(np.float32).reshape(np.shape(state.get(k, st[f"small/{k}"])))
        return dense_weights(cfg, state)
    small = default_small(cfg)
    for k in meta["small_params"]:
        key = f"small/{k}"
        if key not in st:
            continue
        val = st[key].astype(np.float32)
        if k in ("skip_weights", "skip_gates"):
            small[k] = val
        elif k.startswith("blocks."):
            parts = k.split(".")
            i = int(parts[1])
            field = {"attn_scale": "attn_scale", "mlp_scale": "mlp_scale", "resid_mix": "resid_mix", "q_gain": "q_gain"}.get(parts[-1])
            if field is not None:
                small[field][i] = val
    qo, kvb = banks["qo_bank"], banks["kv_bank"]
    return ModelWeights(
        cfg,
        banks["tok_emb.weight"][0],
        qo[:L], kvb[:L], kvb[L:], qo[L:],
        banks["mlp_up_bank"], banks["mlp_down_bank"], small,
    )
