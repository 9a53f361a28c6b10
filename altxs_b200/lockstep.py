"""Lockstep fingerprint of an encode run, carried in the payload.

Encoder and decoder must run the same arithmetic: the same model and weights,
the same linear-layer path (tensor cores or CUDA cores: they differ in the
last bits of the logits), the same CDF rule and precision, the same context
mode and the same update (retrain mode, its schedule and hyper-parameters).
The reference leaves these to the caller's configuration and environment,
and a mismatch desyncs the decoder silently (its config fields and
XSA_* switches, altxs src/xsa_ttt/config.py:271-420).  Here the encoder
writes a fingerprint of all of them in front of the segments and the decoder
refuses a payload whose fingerprint differs from its own, naming the
settings that differ.

Payload layout: an optional header frame, then the reference's framing
``<u64 LE len><segment bytes>`` per segment (incremental.py:1721-1722).  The
header frame's length word has its top bit set (no segment is 2^63 bytes), so
it cannot be mistaken for a segment: ``<u64 LE 2^63 | n><n bytes>`` with the
n bytes = ``b"AXB2"``, u16 format version, 32-byte SHA-256 fingerprint, then a
UTF-8 JSON summary of the settings (for the error message).  Payloads without
the header decode as before, unchecked.
"""

from __future__ import annotations

import dataclasses
import hashlib
import json
import struct

import numpy as np

MAGIC = b"AXB2"
VERSION = 1
HEADER_FLAG = 1 << 63
# Bumped whenever a kernel change alters any result bit of the step or the
# updates, so that payloads of an older build are refused rather than desynced.
NUMERICS = 3


class LockstepMismatch(ValueError):
    """The payload was encoded with settings that differ from the decoder's."""


def weights_digest(packed: dict, small: dict) -> str:
    """SHA-256 of a model's packed weights and small parameters (host arrays)."""
    h = hashlib.sha256()
    for name, p in sorted(packed.items()):
        h.update(name.encode())
        for a in (p.codes, p.row_off8, p.gdesc, p.lut, p.glut):
            if a is not None:
                h.update(np.ascontiguousarray(a).tobytes())
    for k in sorted(small):
        h.update(k.encode())
        h.update(np.ascontiguousarray(small[k], dtype=np.float32).tobytes())
    return h.hexdigest()


def run_settings(dm, online_retrain_enabled: bool) -> dict:
    """Everything that changes the coded bits, as a JSON-able dict."""
    cfg = dm.cfg
    d = {f.name: getattr(cfg, f.name) for f in dataclasses.fields(cfg)}
    d["linear_path"] = "tensor_cores" if dm.tensor_cores else "cuda_cores"
    d["full_params"] = bool(dm.full_params)
    d["online_retrain_enabled"] = bool(online_retrain_enabled)
    d["weights_sha256"] = dm.weights_sha256
    d["numerics"] = NUMERICS
    return d


def fingerprint(settings: dict) -> bytes:
    return hashlib.sha256(json.dumps(settings, sort_keys=True, default=str).encode()).digest()


def header_frame(settings: dict) -> bytes:
    body = MAGIC + struct.pack("<H", VERSION) + fingerprint(settings) + json.dumps(
        settings, sort_keys=True, default=str).encode()
    return struct.pack("<Q", HEADER_FLAG | len(body)) + body


def split_header(payload: bytes) -> tuple[dict | None, bytes | None, bytes]:
    """(settings summary, fingerprint, the framed segments) of a payload;
    (None, None, payload) when it carries no header."""
    if len(payload) < 8:
        return None, None, payload
    (w,) = struct.unpack_from("<Q", payload, 0)
    if not w & HEADER_FLAG:
        return None, None, payload
    n = w & ~HEADER_FLAG
    body = payload[8: 8 + n]
    if len(body) != n or body[:4] != MAGIC:
        raise ValueError("malformed payload header")
    (ver,) = struct.unpack_from("<H", body, 4)
    if ver != VERSION:
        raise ValueError(f"payload header version {ver} is not supported (expected {VERSION})")
    fp = bytes(body[6:38])
    settings = json.loads(body[38:].decode())
    return settings, fp, payload[8 + n:]


def check(settings_enc: dict | None, fp_enc: bytes | None, settings_dec: dict) -> None:
    """Raise LockstepMismatch naming the settings the two runs disagree on."""
    if fp_enc is None or fp_enc == fingerprint(settings_dec):
        return
    keys = sorted(set(settings_enc or {}) | set(settings_dec))
    diff = [f"{k}: payload {settings_enc.get(k)!r}, decoder {settings_dec.get(k)!r}"
            for k in keys if (settings_enc or {}).get(k) != settings_dec.get(k)]
    raise LockstepMismatch("payload was encoded with other settings than this decoder's; "
                           + ("; ".join(diff) if diff else "fingerprints differ"))
