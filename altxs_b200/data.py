"""Input streams for the encoder: byte files (V = 256) and BPE token files.

Same file rules as the reference loader (altxs src/xsa_ttt/data.py:37-200):

- a BPE token file is little-endian uint16 token ids; it is recognised by a
  ``.bpe<V>`` name suffix or by its JSON sidecar (``<file>.json``) having
  ``format`` ``xsa_ttt-bpe-v1`` / ``blsmc-bpe-v1``; the vocabulary is the
  sidecar's ``vocab_size``, else the suffix's ``V``, else 4096; the length is
  the sidecar's ``n_tokens``, else half the file size; a sidecar with
  ``encode_pending`` means the dictionary exists but the tokens do not;
- any other file is a byte stream (V = 256) whose length excludes up to two
  trailers at its end, each ``<blob><8-byte tag><u64 LE blob length>``: first a
  ``BLSMETA1`` trailer, then (before it) an ``M3SIDFTR`` trailer.  A trailer
  whose length does not fit is not a trailer.

The symbols then go to ``incremental.compress_full_sha_incremental`` (or the
engine) with ``vocab_size`` set from :class:`CorpusInfo`.
"""

from __future__ import annotations

import json
import re
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

META_TAG = b"BLSMETA1"
M3_TAG = b"M3SIDFTR"
BPE_FORMATS = ("xsa_ttt-bpe-v1", "blsmc-bpe-v1")
_BPE_SUFFIX = re.compile(r"\.bpe(\d+)$")


@dataclass(frozen=True)
class CorpusInfo:
    path: Path
    kind: str  # "bpe_tokens" | "bytes"
    vocab_size: int
    n_symbols: int
    source_bytes: int | None
    meta: dict = field(default_factory=dict)


def sidecar_meta(path: Path) -> dict:
    side = Path(str(path) + ".json")
    return json.loads(side.read_text(encoding="utf8")) if side.is_file() else {}


def _suffix_vocab(path: Path) -> int | None:
    m = _BPE_SUFFIX.search(path.name)
    return int(m.group(1)) if m else None


def _strip_trailer(path: Path, end: int, tag: bytes) -> int:
    """End of the data before a ``<blob><tag><u64 len>`` trailer ending at ``end``."""
    tail_n = len(tag) + 8
    if end < tail_n:
        return end
    with open(path, "rb") as f:
        f.seek(end - tail_n)
        tail = f.read(tail_n)
    if tail[: len(tag)] != tag:
        return end
    blob = int.from_bytes(tail[len(tag):], "little")
    if blob > end - tail_n:
        return end
    return end - tail_n - blob


def byte_stream_length(path: Path) -> int:
    end = path.stat().st_size
    end = _strip_trailer(path, end, META_TAG)
    return _strip_trailer(path, end, M3_TAG)


def describe(path: str | Path) -> CorpusInfo:
    p = Path(path)
    if not p.is_file():
        raise FileNotFoundError(f"input not found: {p}")
    meta = sidecar_meta(p)
    if _suffix_vocab(p) is not None or meta.get("format") in BPE_FORMATS:
        if meta.get("encode_pending"):
            raise FileNotFoundError(f"BPE dictionary present but the tokens are not: {p}")
        vocab = int(meta.get("vocab_size", _suffix_vocab(p) or 4096))
        n = int(meta["n_tokens"]) if meta.get("n_tokens") is not None else p.stat().st_size // 2
        return CorpusInfo(p, "bpe_tokens", vocab, n, meta.get("source_bytes"), meta)
    n = byte_stream_length(p)
    return CorpusInfo(p, "bytes", 256, n, meta.get("source_bytes", n), meta)


def load_symbols(path: str | Path, *, max_symbols: int | None = None,
                 mmap: bool = True) -> tuple[np.ndarray, CorpusInfo]:
    """The stream's symbols (uint16 tokens or uint8 bytes) and its description."""
    info = describe(path)
    n = info.n_symbols if max_symbols is None else min(info.n_symbols, int(max_symbols))
    if info.kind == "bpe_tokens":
        if mmap:
            arr = np.memmap(info.path, dtype="<u2", mode="r")[:n]
        else:
            arr = np.frombuffer(info.path.read_bytes()[: 2 * n], dtype="<u2").copy()
        if arr.size and int(arr.max()) >= info.vocab_size:
            raise ValueError(f"token id {int(arr.max())} outside vocabulary {info.vocab_size}")
        return arr, info
    if mmap:
        arr = np.memmap(info.path, dtype=np.uint8, mode="r")[:n]
    else:
        with open(info.path, "rb") as f:
            arr = np.frombuffer(f.read(n), dtype=np.uint8).copy()
    meta = dict(info.meta)
    file_n = info.path.stat().st_size
    if n < file_n:
        meta["m3_trailer_stripped"] = int(file_n - n)
    return arr, CorpusInfo(info.path, "bytes", 256, int(n), int(n), meta)
