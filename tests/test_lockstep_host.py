"""Host rules of the lockstep header: framing, fingerprint, mismatch report."""

from __future__ import annotations

import struct

import pytest

from altxs_b200 import lockstep


def _settings(**over):
    s = {"cdf_mode": "fixed", "cdf_bits": 20, "linear_path": "tensor_cores", "context_mode": "sliding",
         "retrain_mode": "lora", "weights_sha256": "ab" * 32, "numerics": lockstep.NUMERICS}
    s.update(over)
    return s


def test_header_round_trip_and_segments_follow():
    seg = b"\x01\x02\x03"
    payload = lockstep.header_frame(_settings()) + struct.pack("<Q", len(seg)) + seg
    got, fp, rest = lockstep.split_header(payload)
    assert got == _settings() and fp == lockstep.fingerprint(_settings())
    assert rest == struct.pack("<Q", 3) + seg
    (w,) = struct.unpack_from("<Q", payload, 0)
    assert w >> 63 == 1  # the header's length word can never be a segment length


def test_payload_without_header_passes_unchecked():
    payload = struct.pack("<Q", 2) + b"\x05\x06"
    got, fp, rest = lockstep.split_header(payload)
    assert got is None and fp is None and rest == payload
    lockstep.check(got, fp, _settings())  # nothing to compare against


def test_mismatch_names_the_settings():
    enc = _settings()
    dec = _settings(linear_path="cuda_cores", cdf_bits=16)
    with pytest.raises(lockstep.LockstepMismatch) as e:
        lockstep.check(enc, lockstep.fingerprint(enc), dec)
    msg = str(e.value)
    assert "linear_path" in msg and "cdf_bits" in msg and "cdf_mode" not in msg
    lockstep.check(enc, lockstep.fingerprint(enc), dict(enc))  # equal settings pass


def test_malformed_header_is_refused():
    bad = struct.pack("<Q", (1 << 63) | 10) + b"XXXX" + b"\x00" * 6
    with pytest.raises(ValueError):
        lockstep.split_header(bad)
