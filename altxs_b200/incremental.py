"""Reference-facing entry points: full-stream encode / blind decode.

Same names, arguments, payload framing and result keys as the reference
``compress_full_sha_incremental`` / ``decompress_full_sha_incremental``
(altxs src/xsa_ttt/incremental.py:1561-1779, 1799-1976), so a caller of that
path can switch to this engine.  ``model`` may be a ``ModelWeights``, a
``DeviceModel`` or a path to a v5 mixed-bit codec; ``cfg`` a ``ModelConfig``
(or anything ``ModelConfig.from_reference_cfg`` accepts).  ``row_batch`` and
``verify_end`` are accepted for signature parity like the reference.

The multi-stream forms (``compress_streams`` / ``decompress_streams``) run
many independent streams in lockstep on one GPU; the single-stream entry
points are the n = 1 case.
"""

from __future__ import annotations

import hashlib
import time
from pathlib import Path
from typing import Any

import numpy as np
import torch

from .codec import ModelWeights, read_codec
from .config import ModelConfig
from .engine import DeviceModel, Engine


def _symbols_for_hash(arr: np.ndarray) -> bytes:
    """Stable byte view for SHA (compress.py:99-105): u8 or little-endian u16."""
    if arr.dtype == np.uint8:
        return arr.tobytes()
    return np.asarray(arr, dtype="<u2").tobytes()


def _as_symbol_array(data, vocab_size: int) -> np.ndarray:
    if isinstance(data, (bytes, bytearray, memoryview)):
        if vocab_size > 256:
            raise ValueError("bytes input requires vocab_size <= 256")
        return np.frombuffer(bytes(data), dtype=np.uint8)
    return np.asarray(data, dtype=np.uint8 if vocab_size <= 256 else np.uint16)


def _resolve(model, cfg, device) -> tuple[DeviceModel, ModelConfig]:
    if isinstance(model, DeviceModel):
        dm = model
    else:
        if isinstance(model, (str, Path)):
            model = read_codec(model)
        if not isinstance(model, ModelWeights):
            raise TypeError("model must be ModelWeights, DeviceModel or a codec path")
        if cfg is not None:
            c = cfg if isinstance(cfg, ModelConfig) else ModelConfig.from_reference_cfg(cfg)
            model.cfg = c
        # the full-parameter updates train the model itself: every weight in one arena
        dm = DeviceModel(model, device, full_params=model.cfg.retrain_mode in ("replenish", "full"))
    return dm, dm.cfg


def _make_engine(dm: DeviceModel, online_retrain_enabled: bool, n_total: int | None = None) -> Engine:
    """Engine with the configured update: LoRA adapters, or every weight
    ("replenish" / "full", one stream at a time from the shipped weights)."""
    ttt = None
    mode = dm.cfg.retrain_mode
    if online_retrain_enabled and dm.cfg.lora_enabled:
        from .ttt import LoraTTT

        ttt = LoraTTT(dm)
    elif online_retrain_enabled and mode in ("replenish", "full"):
        from .replenish import ReplenishTTT

        if not dm.full_params:
            raise ValueError(f"retrain_mode={mode!r} needs DeviceModel(full_params=True)")
        ttt = ReplenishTTT(dm, n_total=n_total)
    return Engine(dm, ttt=ttt)


def compress_streams(model, streams, *, cfg=None, device="cuda", online_retrain_enabled=True):
    dm, cfg = _resolve(model, cfg, device)
    eng = _make_engine(dm, online_retrain_enabled)
    arrs = [_as_symbol_array(s, cfg.vocab_size) for s in streams]
    return eng.encode(arrs), eng


def decompress_streams(model, payloads, n_symbols, *, cfg=None, device="cuda", online_retrain_enabled=True):
    dm, cfg = _resolve(model, cfg, device)
    eng = _make_engine(dm, online_retrain_enabled)
    return eng.decode(list(payloads), list(n_symbols)), eng


def compress_full_sha_incremental(
    model,
    data,
    *,
    cfg=None,
    device="cuda",
    online_retrain_enabled: bool = True,
    progress: bool = True,
    verify_decode: bool = False,
    verify_end: bool = False,
    row_batch: int = 1024,
    decoded_path: str | Path | None = None,
) -> dict[str, Any]:
    del row_batch
    do_verify = bool(verify_decode) or bool(verify_end)
    dm, cfg = _resolve(model, cfg, device)
    arr = _as_symbol_array(data, cfg.vocab_size)
    n = int(arr.shape[0])
    every = max(1, int(cfg.online_retrain_every))
    t0 = time.time()
    eng = _make_engine(dm, online_retrain_enabled, n_total=n)
    res = eng.encode([arr])[0]
    src_sha = hashlib.sha256(_symbols_for_hash(arr)).hexdigest()
    rows = []
    for k, seg in enumerate(res.segments):
        end = min(n, (k + 1) * every)
        rows.append({"pos": int(end), "bpb": len(seg) * 8.0 / max(1, end - k * every)})
    dec_sha = sha_ok = first_mismatch = None
    decoded_bytes = None
    if do_verify:
        eng2 = _make_engine(dm, online_retrain_enabled, n_total=n)
        dec = eng2.decode([res.payload], [n])[0].astype(arr.dtype)
        blob = _symbols_for_hash(dec)
        dec_sha = hashlib.sha256(blob).hexdigest()
        mism = np.flatnonzero(dec != arr)
        first_mismatch = int(mism[0]) if mism.size else None
        sha_ok = dec_sha == src_sha and first_mismatch is None
        if decoded_path:
            Path(decoded_path).parent.mkdir(parents=True, exist_ok=True)
            Path(decoded_path).write_bytes(blob)
            decoded_bytes = len(blob)
    payload_bytes = sum(len(s) for s in res.segments)
    bpb = payload_bytes * 8 / max(1, n)
    if progress:
        dt = time.time() - t0
        print(f"[AC b200] {n:,} sym in {dt:.1f}s ({n / max(dt, 1e-9):,.0f} sym/s), bpb={bpb:.4f}", flush=True)
    updates = cfg.lora_enabled or cfg.retrain_mode in ("replenish", "full")
    retrains = (n - 1) // every if (online_retrain_enabled and updates and n > 0) else 0
    ce = getattr(eng.ttt, "ce_history", []) if eng.ttt is not None else []
    return {
        "payload": res.payload,
        "n_bytes": n,
        "n_symbols": n,
        "payload_bytes": payload_bytes,
        "bpb": bpb,
        "bits_per_symbol": bpb,
        "vocab_size": cfg.vocab_size,
        "retrain_count": retrains,
        "retrain_ce_mean": float(np.mean(ce)) if len(ce) else float("nan"),
        "infer_mode": "segmented_incremental_sha",
        "chunk_bpb_rows": rows,
        "sha256": src_sha,
        "decoded_sha256": dec_sha,
        "sha256_ok": sha_ok,
        "roundtrip_ok": sha_ok,
        "first_mismatch": first_mismatch,
        "segment_bytes": every,
        "verify_decode": do_verify,
        "verify_end": False,
        "decoded_path": str(decoded_path) if (decoded_path and do_verify) else None,
        "decoded_bytes": decoded_bytes,
    }


def decompress_full_sha_incremental(
    model,
    payload: bytes,
    n_symbols: int,
    *,
    cfg=None,
    device="cuda",
    online_retrain_enabled: bool = True,
    progress: bool = True,
    decoded_path: str | Path | None = None,
) -> dict[str, Any]:
    dm, cfg = _resolve(model, cfg, device)
    n = int(n_symbols)
    every = max(1, int(cfg.online_retrain_every))
    t0 = time.time()
    eng = _make_engine(dm, online_retrain_enabled, n_total=n)
    dec = eng.decode([payload], [n])[0]
    arr = dec.astype(np.uint8 if cfg.vocab_size <= 256 else np.uint16)
    blob = _symbols_for_hash(arr)
    if decoded_path:
        Path(decoded_path).parent.mkdir(parents=True, exist_ok=True)
        Path(decoded_path).write_bytes(blob)
    if progress:
        dt = time.time() - t0
        print(f"[AC b200 decode] {n:,} sym in {dt:.1f}s ({n / max(dt, 1e-9):,.0f} sym/s)", flush=True)
    updates = cfg.lora_enabled or cfg.retrain_mode in ("replenish", "full")
    retrains = (n - 1) // every if (online_retrain_enabled and updates and n > 0) else 0
    return {
        "n_symbols": n,
        "payload_bytes": len(payload),
        "segments": (n + every - 1) // every,
        "retrain_count": retrains,
        "decoded_sha256": hashlib.sha256(blob).hexdigest(),
        "decoded_path": str(decoded_path) if decoded_path else None,
        "infer_mode": "segmented_incremental_sha",
        "decoded": None if decoded_path else blob,
    }


__all__ = [
    "compress_full_sha_incremental",
    "decompress_full_sha_incremental",
    "compress_streams",
    "decompress_streams",
]
