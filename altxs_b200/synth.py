"""Seeded synthetic inputs: Zipf-Markov symbol streams and mixed-bit weights.

The reference measures on enwik9 (``payload_sim``), which is not available
here; these generators stand in for it with the shapes and distributions the
benchmark configs name:

* symbol streams: an order-2 Markov source whose marginal ranks follow a
  truncated Zipf(alpha) law.  Symbol ``x_t`` is ``(r_t * m + o) mod V`` where
  ``r_t`` is a Zipf rank drawn by inverse CDF and ``(m, o)`` are hashed from
  the previous two symbols (``m`` odd, so the map is a bijection mod 2^k).
  All randomness comes from splitmix64 of (seed, position), so streams are
  reproducible and generated vectorised across many streams at once.
* weights: per 64-wide group along K, a bit width drawn from {2, 3, 4} with
  probabilities {0.25, 0.35, 0.40} (3.15 bits/weight), codes uniform over
  ``[0, 2^b)``, fp16 scales ``|N(0, 0.02)|``, symmetric levels
  ``(code - (2^b - 1)/2) * scale`` (the reference's ``symmetric`` codebook
  mode, altxs ``src/hyperflow_distillation/mixed_bit_delta.py:147-152``).
"""

from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)


def splitmix64(x: np.ndarray) -> np.ndarray:
    """Vectorised splitmix64 finaliser over uint64 arrays (wrapping)."""
    with np.errstate(over="ignore"):
        z = np.asarray(x, dtype=np.uint64) + _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def zipf_cdf(vocab: int, alpha: float = 1.1) -> np.ndarray:
    w = 1.0 / np.power(np.arange(1, vocab + 1, dtype=np.float64), alpha)
    c = np.cumsum(w)
    return c / c[-1]


def zipf_markov(n: int, vocab: int, seeds, alpha: float = 1.1) -> np.ndarray:
    """Streams ``[len(seeds), n]`` (int32) from the order-2 Zipf-Markov source."""
    seeds = np.atleast_1d(np.asarray(seeds, dtype=np.uint64))
    s = seeds.shape[0]
    cdf = zipf_cdf(vocab, alpha)
    pow2 = vocab & (vocab - 1) == 0
    key_u = splitmix64(seeds * np.uint64(0xD1B54A32D192ED03) + np.uint64(1))
    key_h = splitmix64(seeds * np.uint64(0xD1B54A32D192ED03) + np.uint64(2))
    out = np.empty((s, n), dtype=np.int32)
    a = np.zeros(s, dtype=np.uint64)
    b = np.zeros(s, dtype=np.uint64)
    v64 = np.uint64(vocab)
    with np.errstate(over="ignore"):
        for t in range(n):
            u_bits = splitmix64(key_u ^ (np.uint64(t) * _GOLDEN))
            u = (u_bits >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
            r = np.minimum(np.searchsorted(cdf, u, side="right"), vocab - 1).astype(np.uint64)
            h = splitmix64(key_h ^ (a * v64 + b))
            if pow2:
                m = (np.uint64(2) * (h % np.uint64(max(1, vocab // 2)))) + np.uint64(1)
            else:
                m = np.ones_like(h)
            o = (h >> np.uint64(32)) % v64
            x = (r * m + o) % v64
            out[:, t] = x.astype(np.int32)
            a, b = b, x
    return out


# ---- synthetic mixed-bit weights -------------------------------------------

BITS_CHOICES = np.array([2, 3, 4], dtype=np.uint8)
BITS_PROBS = np.array([0.25, 0.35, 0.40])
GROUP = 64


def synth_groups(rows: int, cols: int, rng: np.random.Generator):
    """Random mixed-bit groups for a ``[rows, cols]`` matrix (groups along cols).

    Returns ``bits [rows, G] u8``, ``codes [rows, cols] u8``,
    ``scales [rows, G] fp16``.
    """
    if cols % GROUP:
        raise ValueError("cols must be a multiple of 64")
    g = cols // GROUP
    bits = rng.choice(BITS_CHOICES, size=(rows, g), p=BITS_PROBS).astype(np.uint8)
    raw = rng.integers(0, 1 << 16, size=(rows, cols), dtype=np.uint32)
    nlev = (np.uint32(1) << np.repeat(bits, GROUP, axis=1).astype(np.uint32))
    codes = (raw % nlev).astype(np.uint8)
    scales = np.abs(rng.normal(0.0, 0.02, size=(rows, g))).astype(np.float16)
    return bits, codes, scales


def dequant_symmetric(bits: np.ndarray, codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Dense fp32 values of symmetric groups (reference ``_symmetric_levels``)."""
    rows, cols = codes.shape
    b = np.repeat(bits, GROUP, axis=1).astype(np.float32)
    center = (np.power(2.0, b, dtype=np.float32) - np.float32(1.0)) / np.float32(2.0)
    lev = codes.astype(np.float32) - center
    s = np.repeat(scales.astype(np.float32), GROUP, axis=1)
    out = lev * s
    out[b == 0] = 0.0
    return out.astype(np.float32)
