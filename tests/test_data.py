"""Input-stream rules: byte files with trailers, BPE token files with sidecars."""

from __future__ import annotations

import json

import numpy as np
import pytest

from altxs_b200.data import M3_TAG, META_TAG, describe, load_symbols


def _trailer(tag: bytes, blob: bytes) -> bytes:
    return blob + tag + len(blob).to_bytes(8, "little")


def test_plain_bytes(tmp_path):
    p = tmp_path / "stream.bin"
    p.write_bytes(bytes(range(200)))
    arr, info = load_symbols(p)
    assert info.kind == "bytes" and info.vocab_size == 256 and info.n_symbols == 200
    assert np.array_equal(arr, np.arange(200, dtype=np.uint8))


def test_bytes_with_both_trailers(tmp_path):
    body = np.random.default_rng(0).integers(0, 256, 1000, dtype=np.uint8).tobytes()
    p = tmp_path / "product"
    p.write_bytes(body + _trailer(M3_TAG, b"m3" * 20) + _trailer(META_TAG, b"{meta}"))
    arr, info = load_symbols(p, mmap=False)
    assert info.n_symbols == 1000 and arr.tobytes() == body
    assert info.meta["m3_trailer_stripped"] == p.stat().st_size - 1000


def test_bad_trailer_length_is_data(tmp_path):
    p = tmp_path / "odd"
    data = b"x" * 10 + META_TAG + (10 ** 6).to_bytes(8, "little")
    p.write_bytes(data)
    assert describe(p).n_symbols == len(data)


def test_bpe_by_suffix(tmp_path):
    toks = np.random.default_rng(1).integers(0, 4096, 777).astype("<u2")
    p = tmp_path / "corpus.bpe4096"
    p.write_bytes(toks.tobytes())
    arr, info = load_symbols(p)
    assert info.kind == "bpe_tokens" and info.vocab_size == 4096 and info.n_symbols == 777
    assert np.array_equal(arr, toks)


def test_bpe_by_sidecar(tmp_path):
    toks = np.random.default_rng(2).integers(0, 1000, 500).astype("<u2")
    p = tmp_path / "tokens.bin"
    p.write_bytes(toks.tobytes())
    (tmp_path / "tokens.bin.json").write_text(json.dumps(
        {"format": "xsa_ttt-bpe-v1", "vocab_size": 1000, "n_tokens": 300, "source_bytes": 1234}))
    arr, info = load_symbols(p, max_symbols=250)
    assert info.kind == "bpe_tokens" and info.vocab_size == 1000 and info.n_symbols == 300
    assert info.source_bytes == 1234 and len(arr) == 250 and np.array_equal(arr, toks[:250])


def test_bpe_pending_and_range(tmp_path):
    p = tmp_path / "c.bpe512"
    p.write_bytes(np.array([1, 2, 600], dtype="<u2").tobytes())
    with pytest.raises(ValueError):
        load_symbols(p)
    (tmp_path / "c.bpe512.json").write_text(json.dumps({"encode_pending": True}))
    with pytest.raises(FileNotFoundError):
        describe(p)
