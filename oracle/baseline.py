"""Timed CPU baseline: the reference's eager fp32 decode path, restated.

Test and CPU-baseline infrastructure only (see ``oracle/__init__.py``).  Used by
``bench.py`` for its ``cpu_baseline`` leg and for ``--impl reference``: one
stream of the benchmark workload (33M model, full ``ctx`` window) is decoded
symbol by symbol on the host cores with the torch fp32 step
(``oracle/model.py``) and the C coder (``oracle/coder.c``) -- the same work
per symbol as the reference's eager ``StaticACEngine`` W=1 decode
(altxs src/xsa_ttt/incremental.py:1463-1550 with XSA_AC_FUSED=0,
XSA_AC_GPU_AC=0): model step over the window, softmax -> integer masses,
range-decode one symbol.  The bitstream it decodes is produced first by the
same oracle (untimed), and the decoded symbols are checked.
"""

from __future__ import annotations

import os
import time

import numpy as np
import torch

from altxs_b200.codec import ModelWeights
from altxs_b200.synth import zipf_markov
from oracle.coder import IncrementalDecoder, IncrementalEncoder, cum_from_logits
from oracle.model import OracleLoRA, OracleModel, OracleWeights


def cpu_decode_baseline(weights: ModelWeights, *, target_s: float = 10.0, max_symbols: int = 4096,
                        seed: int = 1, threads: int | None = None) -> dict:
    cfg = weights.cfg
    threads = int(threads or os.cpu_count() or 1)
    torch.set_num_threads(threads)
    om = OracleModel(OracleWeights.from_model_weights(weights))
    lora = OracleLoRA.init(cfg) if cfg.lora_enabled else None
    n_pre = cfg.ctx

    def cum_of(lg):
        return cum_from_logits(lg.numpy()[None], cfg.cdf_mode, cfg.cdf_bits)[0]

    # calibrate: how many symbols fit in target_s
    data = zipf_markov(n_pre + max_symbols + 1, cfg.vocab_size, [seed])[0]
    st = om.new_stream()
    lg = om.prefill(st, data[:n_pre], lora)
    t0 = time.perf_counter()
    probe = 4
    for t in range(probe):
        cum_of(lg)
        lg = om.step(st, int(data[n_pre + t]), lora)
    per = (time.perf_counter() - t0) / probe
    n = int(max(8, min(max_symbols, target_s / max(per, 1e-6))))
    # encode (untimed) the sample
    st = om.new_stream()
    lg = om.prefill(st, data[:n_pre], lora)
    enc = IncrementalEncoder(n * 8 + 64)
    for t in range(n):
        s = int(data[n_pre + t])
        enc.encode(cum_of(lg), s)
        if t + 1 < n:
            lg = om.step(st, s, lora)
    payload = enc.finish()
    # decode (timed)
    st = om.new_stream()
    lg = om.prefill(st, data[:n_pre], lora)
    dec = IncrementalDecoder(payload)
    out = np.empty(n, dtype=np.int64)
    t0 = time.perf_counter()
    for t in range(n):
        s = dec.decode(cum_of(lg))
        out[t] = s
        if t + 1 < n:
            lg = om.step(st, s, lora)
    dt = time.perf_counter() - t0
    if not np.array_equal(out, data[n_pre: n_pre + n]):
        raise RuntimeError("CPU baseline round trip failed")
    return {
        "value": n / dt,
        "unit": "sym/s",
        "cores": threads,
        "kind": "port",
        "sample": f"1 stream, {n} symbols decoded after a {n_pre}-token prefill (full window), "
                  f"torch fp32 step + C range coder, {len(payload) * 8 / n:.3f} bits/symbol",
        "seconds": dt,
        "bits_per_symbol": len(payload) * 8 / n,
    }
