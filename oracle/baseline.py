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


# ---------------------------------------------------------------------------
# Aggregate CPU baseline: one process per host core, each decoding its own
# streams single-threaded.


def _ref_import(ref_root: str):
    """The reference's own modules from an installed copy (eager CPU path:
    XSA_AC_FUSED=0, XSA_AC_GPU_AC=0, XSA_AC_GRAPH=0; one-symbol windows,
    XSA_AC_WINDOW=1, so encode runs decode's exact op sequence)."""
    import sys

    os.environ.update(XSA_AC_FUSED="0", XSA_AC_GPU_AC="0", XSA_AC_GRAPH="0", XSA_AC_WINDOW="1")
    for p in (ref_root, os.path.join(ref_root, "model")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import xsa_ttt.incremental as inc
    from xsa_ttt.config import XsaTttConfig
    from xsa_ttt.model import GPT

    return inc, XsaTttConfig, GPT


def reference_xsa_config(cfg, XsaTttConfig):
    """The reference's config for this engine's plain GPT: every motif off,
    tied embeddings (src/xsa_ttt/config.py field names)."""
    h = XsaTttConfig(seed=cfg.seed)
    for k in ("vocab_size", "num_layers", "model_dim", "num_heads", "num_kv_heads", "mlp_mult",
              "rope_base", "rope_dims", "qk_gain_init", "logit_softcap", "ln_scale",
              "skip_gates_enabled", "block_size", "online_retrain_every", "grad_clip"):
        setattr(h, k, getattr(cfg, k))
    for k in ("xsa_last_n", "num_loops", "parallel_start_layer"):
        setattr(h, k, 0)
    for k in ("smear_gate_enabled", "sparse_attn_gate_enabled", "attn_out_gate_enabled",
              "gated_attn_enabled", "asym_logit_rescale", "rope_yarn", "gradient_checkpointing"):
        setattr(h, k, False)
    h.tie_embeddings = True
    return h


def _worker(wid: int, spec: dict, barrier, queue) -> None:
    """One single-threaded decoder process: its share of the streams, each
    decoded from symbol ``start`` with the ``start`` preceding symbols as
    context; the timed part is the per-symbol decode (the context prefill
    that opens the segment is measured and left out)."""
    import sys

    sys.path.insert(0, spec["repo_root"])
    torch.set_num_threads(1)
    from altxs_b200 import codec as C
    from altxs_b200.config import c3_config

    out = {"wid": wid, "n": 0, "steps": 0, "decode_s": 0.0, "bytes": {}, "ok": True, "err": None}
    try:
        cfg = c3_config()
        w = C.synth_weights(cfg, seed=spec["weight_seed"])
        start, n = int(spec["start"]), int(spec["n_symbols"])
        if spec["ref_root"]:
            inc, XsaTttConfig, GPT = _ref_import(spec["ref_root"])
            h = reference_xsa_config(cfg, XsaTttConfig)
            h.online_retrain_every = n  # one segment per sample: the static cache holds start + n rows
            torch.manual_seed(0)
            m = GPT(h)
            sd = m.state_dict()
            for k, v in w.dense().items():
                sd[k] = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32))
            m.load_state_dict(sd, strict=True)
            m.eval()
            eng = inc.StaticACEngine(m, h, torch.device("cpu"))
            pre = {"s": 0.0}
            reset = eng.reset_segment

            def timed_reset(prefix, st):
                t = time.perf_counter()
                reset(prefix, st)
                pre["s"] += time.perf_counter() - t

            eng.reset_segment = timed_reset

            def run(arr):
                payload = inc._encode_segment_incremental(eng, arr, arr[start:start + n], start=start)
                pre["s"] = 0.0
                t0 = time.perf_counter()
                dec = inc._decode_segment_incremental(eng, arr, payload, start=start, n_seg=n)
                dt = time.perf_counter() - t0 - pre["s"]
                return payload, np.asarray(dec, dtype=np.int64), dt
        else:
            om = OracleModel(OracleWeights.from_model_weights(w))

            def cum_of(lg):
                return cum_from_logits(lg.numpy()[None], cfg.cdf_mode, cfg.cdf_bits)[0]

            def run(arr):
                st = om.new_stream()
                lg = om.prefill(st, arr[:start])
                enc = IncrementalEncoder(n * 8 + 64)
                for t in range(n):
                    enc.encode(cum_of(lg), int(arr[start + t]))
                    if t + 1 < n:
                        lg = om.step(st, int(arr[start + t]))
                payload = enc.finish()
                st = om.new_stream()
                lg = om.prefill(st, arr[:start])
                dec = IncrementalDecoder(payload)
                got = np.empty(n, dtype=np.int64)
                t0 = time.perf_counter()
                for t in range(n):
                    got[t] = dec.decode(cum_of(lg))
                    if t + 1 < n:
                        lg = om.step(st, int(got[t]))
                return payload, got, time.perf_counter() - t0

        barrier.wait(timeout=600)
        t_loop = time.perf_counter()
        for seed in spec["seeds"]:
            arr = zipf_markov(start + n, cfg.vocab_size, [seed])[0].astype(np.uint16)
            payload, got, dt = run(arr)
            if not np.array_equal(got, arr[start:start + n].astype(np.int64)):
                out["ok"] = False
            out["n"] += n
            out["steps"] += n - 1  # the first symbol's distribution comes from the context prefill
            out["decode_s"] += dt
            out["bytes"][int(seed)] = len(payload)
            if time.perf_counter() - t_loop >= spec["target_s"]:
                break
    except Exception as e:  # reported by the parent
        out["ok"] = False
        out["err"] = f"{type(e).__name__}: {e}"[:300]
    queue.put(out)


def parallel_decode_baseline(*, weight_seed: int, stream_seeds, start: int, n_symbols: int,
                             target_s: float = 10.0, workers: int | None = None,
                             ref_root: str | None = None, repo_root: str | None = None) -> dict:
    """Aggregate decode rate of the host cores: ``workers`` processes (default:
    one per core this process may run on, at most one per GiB of free memory),
    each single-threaded, each decoding whole streams of ``stream_seeds``
    (dealt round-robin) until ``target_s`` of its own wall time has passed.
    With ``ref_root`` the decoder is the reference's own eager CPU path
    (``StaticACEngine`` + ``_encode_segment_incremental`` /
    ``_decode_segment_incremental``, incremental.py:203,1340,1463; kind
    "reference"), otherwise this directory's port (torch fp32 step + C coder;
    kind "port").  value = sum over workers of symbols / decode seconds
    (the workers run concurrently, one per core)."""
    import multiprocessing as mp

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    if workers is None:
        workers = cores
        try:
            import psutil

            workers = max(1, min(workers, int(psutil.virtual_memory().available // (1 << 30))))
        except Exception:
            pass
    seeds = [int(s) for s in stream_seeds]
    workers = max(1, min(int(workers), len(seeds)))
    ctx = mp.get_context("spawn")
    barrier = ctx.Barrier(workers)
    queue = ctx.Queue()
    repo_root = repo_root or os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    procs = []
    for i in range(workers):
        spec = {"repo_root": repo_root, "ref_root": ref_root, "weight_seed": int(weight_seed),
                "seeds": seeds[i::workers], "start": int(start), "n_symbols": int(n_symbols),
                "target_s": float(target_s)}
        p = ctx.Process(target=_worker, args=(i, spec, barrier, queue), daemon=True)
        p.start()
        procs.append(p)
    res = [queue.get(timeout=1800) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    errs = [r["err"] for r in res if r["err"]]
    if errs:
        raise RuntimeError(f"CPU baseline worker failed: {errs[0]}")
    if not all(r["ok"] for r in res):
        raise RuntimeError("CPU baseline round trip failed")
    n_tot = sum(r["n"] for r in res)
    value = sum(r["steps"] / r["decode_s"] for r in res if r["decode_s"] > 0)
    nbytes = {}
    for r in res:
        nbytes.update(r["bytes"])
    kind = "reference" if ref_root else "port"
    what = ("the reference's own eager CPU decode (StaticACEngine, one-symbol windows)" if ref_root
            else "the port of the reference's eager decode (torch fp32 step + C range coder)")
    return {
        "value": value,
        "unit": "sym/s",
        "cores": workers,
        "kind": kind,
        "sample": f"{workers} single-threaded processes, {len(nbytes)} streams x {n_symbols} symbols "
                  f"({n_tot} decoded) from position {start} with the {start} preceding symbols as context, "
                  f"{what}; per-symbol decode timed, the context prefill measured and left out",
        "bits_per_symbol": 8.0 * sum(nbytes.values()) / max(1, n_tot),
        "stream_bytes": nbytes,
        "symbols": n_tot,
    }
