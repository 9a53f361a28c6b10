"""ctypes wrapper over ``oracle/coder.c`` (the CPU coder/CDF restatement).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Reference behaviour restated (altxs project paths):
  * ``src/model/arithmetic_coder_lm.py:49-64``  probs -> integer masses
  * ``src/model/arithmetic_coder_lm.py:90-137`` renorm, bit packing, bit reader
  * ``src/model/arithmetic_coder_lm.py:140-284`` encode / decode loops
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_SO = _HERE / "_build" / "liboracle_coder.so"
_LIB = None


def build() -> Path:
    """Compile ``coder.c`` with the committed Makefile (idempotent)."""
    src = _HERE / "coder.c"
    if not _SO.exists() or _SO.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _SO


def _lib():
    global _LIB
    if _LIB is None:
        build()
        lib = ctypes.CDLL(str(_SO))
        i64, i32, vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p
        lib.oc_encode_cum.restype = i64
        lib.oc_encode_cum.argtypes = [i64, i32, vp, vp, vp, i64]
        lib.oc_decode_cum.restype = i64
        lib.oc_decode_cum.argtypes = [i64, i32, vp, vp, i64, vp]
        lib.oc_cum_from_probs_ref.restype = None
        lib.oc_cum_from_probs_ref.argtypes = [i64, i32, vp, vp]
        lib.oc_cum_from_logits_fixed.restype = ctypes.c_int
        lib.oc_cum_from_logits_fixed.argtypes = [i64, i32, vp, i32, vp]
        lib.oc_cum_from_logits_ref.restype = ctypes.c_int
        lib.oc_cum_from_logits_ref.argtypes = [i64, i32, vp, vp]
        lib.oc_dec_begin.restype = None
        lib.oc_dec_begin.argtypes = [vp, vp, i64]
        lib.oc_dec_next.restype = i32
        lib.oc_dec_next.argtypes = [vp, i32, vp]
        lib.oc_enc_begin.restype = None
        lib.oc_enc_begin.argtypes = [vp, vp, i64]
        lib.oc_enc_next.restype = ctypes.c_int
        lib.oc_enc_next.argtypes = [vp, i32, vp, i32]
        lib.oc_enc_finish.restype = i64
        lib.oc_enc_finish.argtypes = [vp]
        lib.oc_dec_state_size.restype = i64
        lib.oc_enc_state_size.restype = i64
        _LIB = lib
    return _LIB


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def cum_from_probs_ref(probs: np.ndarray) -> np.ndarray:
    """``max(1, floor(p*1e6+0.5))`` masses -> cum tables ``[n, V+1]`` (u64)."""
    p = np.ascontiguousarray(probs, dtype=np.float32)
    if p.ndim == 1:
        p = p[None]
    n, v = p.shape
    cum = np.empty((n, v + 1), dtype=np.uint64)
    _lib().oc_cum_from_probs_ref(n, v, _ptr(p), _ptr(cum))
    return cum


def cum_from_logits(logits: np.ndarray, mode: str = "fixed", cdf_bits: int = 20) -> np.ndarray:
    """Framework CDF rules over softcapped fp32 logits -> cum ``[n, V+1]``."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    if lg.ndim == 1:
        lg = lg[None]
    n, v = lg.shape
    cum = np.empty((n, v + 1), dtype=np.uint64)
    if mode == "fixed":
        rc = _lib().oc_cum_from_logits_fixed(n, v, _ptr(lg), int(cdf_bits), _ptr(cum))
    elif mode == "ref":
        rc = _lib().oc_cum_from_logits_ref(n, v, _ptr(lg), _ptr(cum))
    else:
        raise ValueError(f"unknown cdf mode {mode!r}")
    if rc != 0:
        raise ValueError(f"cdf rule failed (rc={rc})")
    return cum


def encode_cum(cum: np.ndarray, syms: np.ndarray) -> bytes:
    """Encode ``syms`` with one cum row per symbol; returns the packed bytes."""
    c = np.ascontiguousarray(cum, dtype=np.uint64)
    s = np.ascontiguousarray(syms, dtype=np.int32)
    n = int(s.shape[0])
    v = int(c.shape[1]) - 1
    if c.shape[0] != n:
        raise ValueError("one cum row per symbol required")
    cap = n * 8 + 64
    out = np.zeros(cap, dtype=np.uint8)
    nbits = _lib().oc_encode_cum(n, v, _ptr(c), _ptr(s), _ptr(out), cap)
    if nbits < 0:
        raise ValueError(f"oracle encode failed (status {-nbits})")
    return out[: (nbits + 7) // 8].tobytes()


def decode_cum(cum: np.ndarray, payload: bytes, n: int) -> np.ndarray:
    c = np.ascontiguousarray(cum, dtype=np.uint64)
    v = int(c.shape[1]) - 1
    buf = np.frombuffer(bytes(payload) + b"\0", dtype=np.uint8).copy()
    out = np.empty(int(n), dtype=np.int32)
    rc = _lib().oc_decode_cum(int(n), v, _ptr(c), _ptr(buf), len(payload), _ptr(out))
    if rc != 0:
        raise ValueError(f"oracle decode failed (status {-rc})")
    return out


def encode_probs(probs: np.ndarray, syms: np.ndarray) -> bytes:
    """Reference-rule encode: probs rows -> masses -> bitstream."""
    return encode_cum(cum_from_probs_ref(probs), syms)


def decode_probs(probs: np.ndarray, payload: bytes, n: int) -> np.ndarray:
    return decode_cum(cum_from_probs_ref(probs), payload, n)


class IncrementalEncoder:
    """One symbol per call, for model-in-the-loop coding on the CPU."""

    def __init__(self, capacity_bytes: int):
        L = _lib()
        self._st = ctypes.create_string_buffer(int(L.oc_enc_state_size()))
        self._out = np.zeros(int(capacity_bytes), dtype=np.uint8)
        L.oc_enc_begin(self._st, _ptr(self._out), self._out.size)

    def encode(self, cum_row: np.ndarray, sym: int) -> None:
        c = np.ascontiguousarray(cum_row, dtype=np.uint64)
        rc = _lib().oc_enc_next(self._st, c.shape[0] - 1, _ptr(c), int(sym))
        if rc != 0:
            raise ValueError(f"oracle encode failed (status {-rc})")

    def finish(self) -> bytes:
        nbits = _lib().oc_enc_finish(self._st)
        if nbits < 0:
            raise ValueError(f"oracle encode failed (status {-nbits})")
        return self._out[: (nbits + 7) // 8].tobytes()


class IncrementalDecoder:
    def __init__(self, payload: bytes):
        L = _lib()
        self._st = ctypes.create_string_buffer(int(L.oc_dec_state_size()))
        self._buf = np.frombuffer(bytes(payload) + b"\0" * 8, dtype=np.uint8).copy()
        L.oc_dec_begin(self._st, _ptr(self._buf), len(payload))

    def decode(self, cum_row: np.ndarray) -> int:
        c = np.ascontiguousarray(cum_row, dtype=np.uint64)
        s = _lib().oc_dec_next(self._st, c.shape[0] - 1, _ptr(c))
        if s < 0:
            raise ValueError("oracle decode failed (bad CDF total)")
        return int(s)


__all__ = [
    "IncrementalEncoder",
    "IncrementalDecoder",
    "build",
    "cum_from_probs_ref",
    "cum_from_logits",
    "encode_cum",
    "decode_cum",
    "encode_probs",
    "decode_probs",
]
