#!/usr/bin/env python
"""Benchmark: decode symbols/sec of the 33M, 3.15-bpw model-and-code loop.

Workload (the reference's "box-scale sharded run" configuration): 2048 independent streams
split evenly over N GPUs (one process per GPU), the 33M model (8L/512d/8h,
MLP 2048, V 16384) with seeded random mixed 2/3/4-bit weights, sliding
window filled to 2048 of 2048, symbols from the seeded Zipf-Markov source.
A step decodes one symbol for every stream on every GPU: model step over the
full window, logits -> integer CDF, range decode.  The LoRA schedule runs
inside the timed steps: segment boundaries every 16,384 symbols per stream,
staggered over the streams, each one a coder reload plus a test-time update
over the stream's last 2048 symbols.  Streams share no data, so
there is no collective on the hot path (weak per-stream work, fixed total
streams -> "strong" scaling); NCCL only gathers per-stream byte counts.

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
cuda synchronize, CUDA events on the launch stream, max over ranks.  Each
step replays the decode step from a CUDA graph (captured on its first calls);
updates and segment reloads launch eagerly in between.  The KV windows
(~103 GB per GPU at N=1) are far larger than L2, so every step streams its
inputs from HBM.  The per-kernel breakdown and the attention roofline come
from re-running the same K steps launch by launch with CUDA events around
every launch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference|reference-triton]

--impl reference times the CPU port of the reference's eager decode on the host
cores; --impl reference-triton times the reference's own GPU decode (its Triton
megakernel and GPU coder, from the offline install in baseline/_ref) on one GPU.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode symbols/sec (33M, 3.15 bpw)"
GLOBAL_STREAMS = 2048
WEIGHT_SEED = 1234


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference", "reference-triton"), default="b200")
    ap.add_argument("--ref-symbols", type=int, default=REF_TRITON_SYMBOLS,
                    help="stream length of the reference-triton arm")
    ap.add_argument("--streams", type=int, default=GLOBAL_STREAMS, help="global stream count")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--fill", choices=("prefill", "random"), default="prefill",
                    help="how the windows are filled before timing: code the preceding 2048 symbols "
                         "(default) or write seeded random K/V rows (profiling runs: same per-step work, "
                         "no 2048-step warm-up)")
    ap.add_argument("--cuda-cores", action="store_true",
                    help="run the step's linear layers on CUDA cores from the packed codes (the few-stream "
                         "choice: 0.43 bytes per weight read per step instead of the 4-byte tensor-core planes)")
    ap.add_argument("--packed", type=int, default=None,
                    help="1: the step's tensor-core linears expand the packed codes in the GEMM; 0: they read "
                         "the dense hi/lo planes (same bits); default: the library's setting")
    ap.add_argument("--fusion", action="store_true",
                    help="with --cuda-cores and at most 4 streams per GPU: run each step as one fused "
                         "persistent kernel instead of a kernel per phase (same bits; measured slower)")
    ap.add_argument("--replenish", action="store_true",
                    help="instead of the decode benchmark: one full-parameter replenish boundary of the 33M "
                         "model (Forward-XM: gradient of every weight over an 18,432-token window, AdamW, "
                         "four candidate updates each scored on an 18,432-token probe window), one JSON line")
    ap.add_argument("--lora-update", action="store_true",
                    help="instead of the decode benchmark: one test-time LoRA boundary update (33M model, full "
                         "window), for 1 and for --update-rows streams, one JSON line each")
    ap.add_argument("--update-rows", type=int, default=8)
    ap.add_argument("--attention", action="store_true",
                    help="instead of the decode benchmark: the window attention kernel at the 33M window shape "
                         "and the reset-mode context prefill with it and with the materialised attention")
    ap.add_argument("--c2", action="store_true",
                    help="instead of the decode benchmark: the linear-layer microbenchmark (the C3 layer "
                         "shapes K x N at M = 1, 16, 128, 512 rows, tensor-core and CUDA-core paths), one "
                         "JSON line per case")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    return rank, world, local


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms (read-only)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(gpu_index), "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
            "power_w_max": max(power) if power else None,
        }


def cpu_parallel(args, stream_seeds, n_symbols: int, target_s: float) -> dict:
    """Aggregate CPU decode rate over the host cores (one single-threaded
    process per core, each decoding whole streams of the benchmark workload):
    the reference's own eager CPU path from the offline install when it is
    there, else the port under oracle/."""
    from altxs_b200.config import c3_config
    from oracle.baseline import parallel_decode_baseline

    ref_root = str(REF_INSTALL) if (REF_INSTALL / "xsa_ttt").is_dir() else None
    return parallel_decode_baseline(weight_seed=WEIGHT_SEED, stream_seeds=stream_seeds, start=c3_config().ctx,
                                    n_symbols=n_symbols, target_s=target_s, ref_root=ref_root,
                                    repo_root=str(ROOT))


def run_reference(args, rank, world):
    """CPU reference arm: the reference's eager decode on every host core
    (one process per core, each decoding its own streams of the workload:
    window full, the chunk of W + K symbols each stream decodes in the GPU
    arm).  Rank 0 runs it; other ranks exit."""
    if rank != 0:
        return
    t0 = time.perf_counter()
    chunk = max(3, args.warmup) + max(1, args.steps)
    res = cpu_parallel(args, list(range(1000, 1000 + args.streams)), chunk, args.cpu_seconds)
    value = float(res["value"])
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "sym/s",
        "n_gpus": world,
        "steps": max(1, args.steps),
        "warmup": max(3, args.warmup),
        "ms_per_step": 1000.0 * res["cores"] / value,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic Zipf-Markov (alpha 1.1), seeded random mixed-bit weights",
        "config": config_block(world, args.streams, args.cuda_cores),
        "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": value, "unit": "sym/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "bits_per_symbol": res["bits_per_symbol"],
        "streams_decoded": len(res["stream_bytes"]),
        "wall_s": time.perf_counter() - t0,
    }
    print(json.dumps(line), flush=True)


REF_INSTALL = ROOT / "baseline" / "_ref"
REF_TRITON_SYMBOLS = 4096


def _ref_xsa_config(cfg, XsaTttConfig):
    """The reference's config for the same model: plain GPT, every motif off,
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


def run_reference_triton(args, rank, world):
    """The reference's own GPU decode on one B200, through its public entry
    points from the offline install in baseline/_ref: the 33M model (dense
    fp32 copy of the same seeded mixed-bit weights), one stream of
    REF_TRITON_SYMBOLS Zipf-Markov symbols encoded with
    ``compress_full_sha_incremental`` and decoded with
    ``decompress_full_sha_incremental`` (src/xsa_ttt/incremental.py:1561,
    :1799) in its stock GPU configuration (Triton fused step, GPU range
    coder, CUDA graphs).  The reference's context
    grows within a segment, so positions 0..4095 attend on average 2048 keys,
    the bench's window.  Updates are off (the reference's lockstep update
    would only lower its rate).  Each step is one full decode call, timed with
    a device synchronize on both sides; the first decode call (Triton
    compilation, graph capture) is a warm-up.  The reference's window switch
    is set to one symbol (``XSA_AC_WINDOW=1``, unless the caller sets it):
    decode steps one row either way, and with it the encoder runs the
    decoder's exact op sequence, so the round trip holds (with 64-symbol
    encode windows the reference's encoder and decoder part within a few
    symbols on this model).  A failure inside the reference prints an
    ``unavailable`` line with the error."""
    if rank != 0:
        return
    os.environ.setdefault("XSA_AC_WINDOW", "1")
    try:
        _run_reference_triton(args)
    except Exception as e:  # the reference's own code failed on this box
        print(json.dumps({"impl": "reference-triton",
                          "unavailable": f"reference GPU decode failed: {type(e).__name__}: {e}"[:400]}))


def _run_reference_triton(args):
    if not (REF_INSTALL / "xsa_ttt").is_dir():
        print(json.dumps({"impl": "reference-triton", "unavailable": "baseline/_ref is not installed"}))
        return
    for p in (REF_INSTALL, REF_INSTALL / "model"):
        sys.path.insert(0, str(p))
    from xsa_ttt.config import XsaTttConfig
    from xsa_ttt.incremental import compress_full_sha_incremental, decompress_full_sha_incremental
    from xsa_ttt.model import GPT

    from altxs_b200 import codec as C
    from altxs_b200.config import c3_config
    from altxs_b200.synth import zipf_markov

    cfg = c3_config()
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    n_sym = args.ref_symbols
    w = C.synth_weights(cfg, seed=WEIGHT_SEED)
    h = _ref_xsa_config(cfg, XsaTttConfig)
    torch.manual_seed(0)
    model = GPT(h)
    sd = model.state_dict()
    for k, v in w.dense().items():
        sd[k] = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32))
    model.load_state_dict(sd, strict=True)
    model = model.to(dev).eval()
    data = zipf_markov(n_sym, cfg.vocab_size, np.array([1000]))[0].astype(np.uint16)

    def sync():
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)

    t0 = time.perf_counter()
    enc = compress_full_sha_incremental(model, data, cfg=h, device=dev, online_retrain_enabled=False,
                                        progress=False)
    sync()
    enc_s = time.perf_counter() - t0
    times, ok = [], True
    for i in range(max(1, args.warmup) + max(1, min(args.steps, 3))):
        sync()
        t1 = time.perf_counter()
        dec = decompress_full_sha_incremental(model, enc["payload"], n_sym, cfg=h, device=dev,
                                              online_retrain_enabled=False, progress=False)
        sync()
        if i >= max(1, args.warmup):
            times.append(time.perf_counter() - t1)
        ok = ok and bool(dec.get("decoded_sha256") == enc.get("sha256"))
    s = float(statistics.median(times))
    value = n_sym / s
    line = {
        "impl": "reference-triton",
        "metric": METRIC,
        "value": value,
        "unit": "sym/s",
        "n_gpus": 1,
        "steps": len(times),
        "warmup": max(1, args.warmup),
        "ms_per_step": 1000.0 * s,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16/f32 (reference stock)",
        "data": "synthetic Zipf-Markov (alpha 1.1), dense copy of the seeded random mixed-bit weights",
        "config": {"workload": f"reference stock GPU decode, 1 stream x {n_sym} symbols, 33M model, "
                               "context grows 0..n (mean 2048 at 4096), updates off, XSA_AC_WINDOW="
                               + os.environ.get("XSA_AC_WINDOW", ""),
                   "streams": 1, "symbols": n_sym, "device": str(dev)},
        "encode_s": enc_s,
        "bits_per_symbol": 8.0 * float(enc["payload_bytes"]) / n_sym,
        "roundtrip_ok": ok,
    }
    print(json.dumps(line), flush=True)


def run_c2(args) -> None:
    """Linear-layer microbenchmark: Y = X W^T for the C3 layer shapes (layer 0
    of the benchmark model's qkv, o, up, down matrices; 3.15-bit mixed-bit
    weights + fp16 group scales) at M rows of N(0,1) activations.  Each timed
    call is one ``altxs_linear_tc`` (tensor cores as in the decode step: hi/lo
    split of X + tcgen05 GEMM expanding the packed weights in its producer
    warps) or ``altxs_linear`` (tensor_planes: the same GEMM on dense hi/lo
    weight planes; CUDA cores: packed-code GEMV/GEMM), CUDA events around the call, L2
    flushed (256 MB written, then read) before every call, median of 20.  Roofline: HBM for
    M <= 64 on the algorithmic bytes K*N*3.40/8 + 2*M*K + 2*M*N (packed weights
    incl. scales, bf16 activations), tensor cores above on 2*M*K*N."""
    import ctypes

    from altxs_b200 import _lib
    from altxs_b200 import codec as C
    from altxs_b200.config import c3_config
    from altxs_b200.engine import DeviceModel

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = c3_config()
    dm = DeviceModel(C.synth_weights(cfg, seed=WEIGHT_SEED), dev)
    L = _lib.lib()
    peaks, kind = load_peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    st = torch.cuda.current_stream().cuda_stream
    for name, K, N in (("qkv", 512, 1536), ("o", 512, 512), ("up", 512, 2048), ("down", 2048, 512)):
        q = dm.q[name]
        for M in (1, 16, 128, 512, 2048):  # the C2 sizes, then the bench's per-GPU batch
            X = torch.randn(M, K, generator=g, device=dev)
            Y = torch.empty(M, N, device=dev)
            wsb = int(max(L.altxs_linear_workspace_bytes(M, K), L.altxs_linear_tc_workspace_bytes(M, N, K)))
            ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
            # tensor: the step's linear (packed codes expanded in the GEMM, K split by layer
            # shape); tensor_planes: the same GEMM streaming dense hi/lo bf16 weight planes
            for path in ("tensor", "tensor_planes", "cuda_core"):
                hi = getattr(dm._split, f"{name}_hi") if path == "tensor_planes" else None
                lo = getattr(dm._split, f"{name}_lo") if path == "tensor_planes" else None

                def call():
                    if path == "tensor":
                        rc = L.altxs_linear_tc(ctypes.byref(getattr(dm.tiles, name)), 0, N, X.data_ptr(), M,
                                               Y.data_ptr(), ws.data_ptr(), wsb, st)
                    else:
                        rc = L.altxs_linear(ctypes.byref(q), hi, lo, 0, N, X.data_ptr(), M, Y.data_ptr(),
                                            ws.data_ptr(), wsb, st)
                    _lib.check(rc, "altxs_linear")

                for _ in range(3):
                    call()
                times = []
                for _ in range(20):
                    # write then read 256 MB: L2 holds none of the operands, and no dirty
                    # lines whose write-back would land inside the timed call
                    flush.zero_()
                    flush.sum()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    call()
                    e1.record()
                    torch.cuda.synchronize()
                    times.append(e0.elapsed_time(e1) / 1000.0)
                t = statistics.median(times)
                alg_bytes = K * N * 3.40 / 8 + 2 * M * K + 2 * M * N
                flops = 2.0 * M * K * N
                if M <= 64:
                    bound, achieved, peak, unit = "hbm", alg_bytes / t / 1e9, peaks["hbm_gbs"], "GB/s"
                else:
                    bound, achieved, peak, unit = "tensor", flops / t / 1e12, peaks["bf16_tflops"], "TFLOP/s"
                print(json.dumps({"c2": True, "matrix": name, "K": K, "N": N, "M": M, "path": path,
                                  "us": t * 1e6, "tflops": flops / t / 1e12, "alg_gbs": alg_bytes / t / 1e9,
                                  "bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                                  "frac": achieved / peak, "peak_source": f"{kind}"}), flush=True)


def run_replenish(args) -> None:
    """One Forward-XM replenish boundary of the 33M model at its own shapes
    (block 2048, segments of 16,384 symbols) on one GPU.  The boundary at
    position 3 x 16,384 trains on the previous segment with its 2048-symbol
    context (18,432 tokens), then scores the candidates W0 + s dW, s in
    0.5, 1, 2, 4, on the just-coded segment (18,432 tokens each).  Timed with
    CUDA events on the launch stream after one warm-up boundary, over --steps
    boundaries (each restarting from the same weights and optimizer state).
    Tensor roofline: algorithmic FLOPs of the four passes (3 x forward for the
    gradient pass, 1 x forward per probe; forward = 2 x parameters x tokens
    + 2 x T^2 x d x layers for causal attention) over the bf16 dense peak;
    the hi/lo operand split issues three MMAs per product, so its ceiling is a
    third of that."""
    import ctypes

    from altxs_b200 import _lib
    from altxs_b200 import codec as C
    from altxs_b200.config import c3_config
    from altxs_b200.engine import DeviceModel
    from altxs_b200.replenish import ReplenishTTT
    from altxs_b200.synth import zipf_markov

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = c3_config()
    cfg.retrain_mode = "replenish"
    cfg.ttt_replenish_warmup_steps = 0
    cfg.ttt_lora_lr = 8e-5
    every, block = cfg.online_retrain_every, cfg.block_size
    dm = DeviceModel(C.synth_weights(cfg, seed=WEIGHT_SEED), dev, full_params=True)
    arr = zipf_markov(3 * every, cfg.vocab_size, [11])[0].astype(np.int32)
    prefix = torch.as_tensor(arr, device=dev)
    ttt = ReplenishTTT(dm, n_total=len(arr))
    peaks, kind = load_peaks()
    L = _lib.lib()
    n_tok = every + block
    T = n_tok - 1
    P = dm.layout.total
    fwd = 2.0 * P * T + 2.0 * T * T * cfg.model_dim * cfg.num_layers
    # time the parts: the gradient pass and one probe forward
    st = torch.cuda.current_stream().cuda_stream
    toks = prefix[every - block: 2 * every].contiguous()

    def call(grad: bool):
        rc = L.altxs_full_loss_grad(ctypes.byref(dm.desc), ctypes.byref(dm.weights_struct),
                                    ctypes.byref(dm.dense_weights()), toks.data_ptr(), n_tok, block - 1,
                                    ttt.loss.data_ptr(), ttt.grad.data_ptr() if grad else None, ttt.ws.data_ptr(),
                                    ttt.ws_bytes, st)
        _lib.check(rc, "altxs_full_loss_grad")

    def timed(fn, reps):
        fn()
        torch.cuda.synchronize()
        out = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            out.append(e0.elapsed_time(e1) / 1000.0)
        return statistics.median(out)

    reps = max(1, min(args.steps, 5))
    t_grad = timed(lambda: call(True), reps)
    t_fwd = timed(lambda: call(False), reps)
    p0, m0, v0 = dm.params.clone(), ttt.m.clone(), ttt.v.clone()

    def boundary():
        dm.params.copy_(p0)
        ttt.m.copy_(m0)
        ttt.v.copy_(v0)
        ttt.step = 0
        dm.refresh()
        ttt.boundary(prefix, 3 * every)

    sampler = ClockSampler(0)
    t_b = timed(boundary, reps)
    clocks = sampler.stop()
    n_cand = len(ttt.xm_last["candidates"])
    flops = 3 * fwd + n_cand * fwd
    tf = flops / t_b / 1e12
    print(json.dumps({
        "replenish": True, "workload": "33M model (8L/512d/8h, MLP 2048, V 16384), block 2048, segment 16384: "
                                       "one Forward-XM boundary, 4 candidates, 1 probe window",
        "tokens_per_window": n_tok, "params": P, "boundary_ms": t_b * 1e3, "grad_pass_ms": t_grad * 1e3,
        "forward_ms": t_fwd * 1e3, "candidates": n_cand, "xm_chosen": ttt.xm_last["chosen"],
        "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": tf / peaks["bf16_tflops"], "peak_source": f"{kind} bf16_tflops",
                     "note": "hi/lo bf16 split: 3 MMAs per product, ceiling 1/3 of peak"},
        "grad_pass_tflops": 3 * fwd / t_grad / 1e12, "forward_tflops": fwd / t_fwd / 1e12,
        "workspace_gib": ttt.ws_bytes / 2 ** 30, "clocks": clocks, "dtype": "f32 math, hi/lo bf16 tensor-core products",
        "data": "synthetic: seeded Zipf-Markov stream, seeded random mixed-bit weights",
    }), flush=True)


def run_attention(args) -> None:
    """Window attention (``altxs_window_attention``: the flash kernel of the
    prefill, the update and the full-parameter forward) and its backward
    (``altxs_window_attention_backward``) at the 33M window (T 2047, 8 heads of
    64), CUDA events around 20 calls each after a warm-up, median; tensor
    roofline on the executed products (3 hi/lo bf16 MMAs per fp32 product:
    6 T^2 hd H flops for the causal half of each of the forward's 2 and the
    backward's 7 products) over the measured bf16 peak.  Then
    one reset-mode context prefill of the 33M model (2047 rows, 8 layers) on
    the flash kernel and on the materialised T x T attention."""
    import ctypes

    from altxs_b200 import _lib
    from altxs_b200 import codec as C
    from altxs_b200.config import c3_config
    from altxs_b200.engine import ContextReset, DeviceModel, StreamBatch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = _lib.lib()
    peaks, kind = load_peaks()
    st = torch.cuda.current_stream().cuda_stream
    for T, H, Hkv, hd in ((2047, 8, 8, 64), (2047, 4, 4, 32)):
        g = torch.Generator(device=dev)
        g.manual_seed(1)
        q = torch.randn(T, H * hd, generator=g, device=dev)
        k = torch.randn(T, Hkv * hd, generator=g, device=dev)
        v = torch.randn(T, Hkv * hd, generator=g, device=dev)
        y = torch.empty(T, H * hd, device=dev)
        wsb = int(L.altxs_window_attention_workspace_bytes(T, H, Hkv, hd))
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)

        def call():
            _lib.check(L.altxs_window_attention(T, H, Hkv, hd, ctypes.c_float(1.0 / hd ** 0.5), q.data_ptr(),
                                                q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                                                y.data_ptr(), y.stride(0), None, ws.data_ptr(), wsb, st),
                       "altxs_window_attention")

        for _ in range(3):
            call()
        times = []
        for _ in range(20):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            call()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        us = statistics.median(times) * 1e3
        flops = 6.0 * T * T * hd * H
        tf = flops / (us / 1e6) / 1e12
        print(json.dumps({"attention": True, "T": T, "H": H, "Hkv": Hkv, "hd": hd, "us": us,
                          "executed_tflops": tf, "frac": tf / peaks["bf16_tflops"],
                          "peak_source": f"{kind} bf16_tflops", "note": "split pass + flash kernel"}), flush=True)
        # the backward from this forward's output and log-sum-exp
        lse = torch.empty(H, T, device=dev)
        _lib.check(L.altxs_window_attention(T, H, Hkv, hd, ctypes.c_float(1.0 / hd ** 0.5), q.data_ptr(),
                                            q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                                            y.data_ptr(), y.stride(0), lse.data_ptr(), ws.data_ptr(), wsb, st),
                   "altxs_window_attention")
        dy = torch.randn(T, H * hd, generator=g, device=dev)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        wbb = int(L.altxs_window_attention_backward_workspace_bytes(T, H, Hkv, hd))
        wsbw = torch.empty(wbb, dtype=torch.uint8, device=dev)

        def bwd():
            _lib.check(L.altxs_window_attention_backward(
                T, H, Hkv, hd, ctypes.c_float(1.0 / hd ** 0.5), q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0),
                v.data_ptr(), v.stride(0), y.data_ptr(), y.stride(0), lse.data_ptr(), dy.data_ptr(), dy.stride(0),
                dq.data_ptr(), dq.stride(0), dk.data_ptr(), dk.stride(0), dv.data_ptr(), dv.stride(0),
                wsbw.data_ptr(), wbb, st), "altxs_window_attention_backward")

        for _ in range(3):
            bwd()
        times = []
        for _ in range(20):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            bwd()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        us = statistics.median(times) * 1e3
        flops = 7 * 3.0 * T * T * hd * H  # S, dP, dq; S^T, dP^T, dk, dv: causal halves, 3 MMAs per product
        tf = flops / (us / 1e6) / 1e12
        print(json.dumps({"attention_backward": True, "T": T, "H": H, "Hkv": Hkv, "hd": hd, "us": us,
                          "executed_tflops": tf, "frac": tf / peaks["bf16_tflops"],
                          "peak_source": f"{kind} bf16_tflops",
                          "note": "split pass + dsum + dk/dv kernel + dq kernel"}), flush=True)
    cfg = dataclasses.replace(c3_config(), context_mode="reset")
    dm = DeviceModel(C.synth_weights(cfg, seed=WEIGHT_SEED), dev, tensor_cores=True)
    b = StreamBatch(dm, 1, words_per_stream=8, hist_len=cfg.ctx + 2)
    b.hist[0, : cfg.ctx] = torch.randint(0, cfg.vocab_size, (cfg.ctx,), device=dev, dtype=torch.int32)
    reset = ContextReset(dm)
    out = {}
    try:
        for on in (1, 0):
            L.altxs_set_flash(on)
            reset(b, [0], cfg.ctx)
            torch.cuda.synchronize()
            times = []
            for _ in range(5):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                reset(b, [0], cfg.ctx)
                e1.record()
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1))
            out["flash" if on else "materialised"] = statistics.median(times)
    finally:
        L.altxs_set_flash(1)
    print(json.dumps({"prefill": True, "rows": cfg.ctx - 1, "layers": cfg.num_layers, "ms": out}), flush=True)


def run_lora_update(args) -> None:
    """One test-time LoRA boundary update of the benchmark's model (33M, rank-8
    q/k/v/o + lm_head adapters) on the full 2047-token window, for 1 and for
    --update-rows streams updated at the same boundary: CUDA events around
    each update after a warm-up, the library's per-class launch profile, and
    the launch count.  Tensor roofline: forward + input-gradient backward
    through the frozen model, 4 x parameters x tokens + attention
    (4 x T^2 x d x layers forward + backward, causal), over the bf16 peak."""
    import ctypes

    from altxs_b200 import _lib
    from altxs_b200 import codec as C
    from altxs_b200.config import c3_config
    from altxs_b200.engine import DeviceModel, StreamBatch
    from altxs_b200.synth import zipf_markov
    from altxs_b200.ttt import LoraTTT

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = c3_config()
    dm = DeviceModel(C.synth_weights(cfg, seed=WEIGHT_SEED), dev, tensor_cores=not args.cuda_cores)
    peaks, kind = load_peaks()
    L = _lib.lib()
    every, ctx = cfg.online_retrain_every, cfg.ctx
    T = ctx - 1
    ncls = len(_lib.KERNEL_CLASSES)
    for rows_n in sorted({1, max(1, args.update_rows)}):
        b = StreamBatch(dm, rows_n, words_per_stream=8, hist_len=ctx + 2)
        data = zipf_markov(ctx + 2, cfg.vocab_size, 1000 + np.arange(rows_n))
        idx = torch.arange(every - ctx - 1, every, device=dev) % b.hist_len
        b.hist[:, idx] = torch.as_tensor(data[:, : ctx + 1].astype(np.int32), device=dev)
        ttt = LoraTTT(dm)
        rows = list(range(rows_n))
        ttt(b, rows, every)  # warm-up (and first AdamW step)
        torch.cuda.synchronize()
        times = []
        for k in range(max(1, min(args.steps, 5))):
            n0 = L.altxs_launch_count()
            if k == 0:
                L.altxs_profile(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            ttt(b, rows, every)
            e1.record()
            torch.cuda.synchronize()
            if k == 0:
                L.altxs_profile(0)
                launches = L.altxs_launch_count() - n0
            times.append(e0.elapsed_time(e1))
        pms = (ctypes.c_double * ncls)()
        pcnt = (ctypes.c_int64 * ncls)()
        L.altxs_profile_read(ncls, pms, pcnt)
        ms = statistics.median(times[1:] if len(times) > 1 else times)
        P = 33554432
        flops = rows_n * (4.0 * P * T + 4.0 * T * T * cfg.model_dim * cfg.num_layers)
        tf = flops / (ms / 1e3) / 1e12
        print(json.dumps({
            "lora_update": True, "rows": rows_n, "window_tokens": T, "ms": ms, "ms_per_row": ms / rows_n,
            "launches": int(launches), "tflops": tf, "frac": tf / peaks["bf16_tflops"],
            "peak_source": f"{kind} bf16_tflops",
            "breakdown_ms": {name: pms[i] for i, name in enumerate(_lib.KERNEL_CLASSES) if pcnt[i]},
            "breakdown_launches": {name: int(pcnt[i]) for i, name in enumerate(_lib.KERNEL_CLASSES) if pcnt[i]},
            "linear": "CUDA cores" if args.cuda_cores else "tensor cores",
        }), flush=True)


def config_block(world: int, streams: int, cuda_cores: bool = False, fusion: bool = False) -> dict:
    return {
        "workload": f"{'box-scale sharded' if streams > 1 else 'single-stream'} decode: {streams} independent "
                    f"stream(s) split over N GPUs, 33M model (8L/512d/8h, MLP 2048, V 16384) at mixed 2/3/4-bit "
                    f"3.15 bpw, ctx 2048 window full",
        "linear": "CUDA cores from the packed codes" if cuda_cores else "tensor cores (hi/lo bf16 planes)",
        "step": ("one fused persistent kernel per step" if cuda_cores and fusion and -(-streams // world) <= 4
                 else "one kernel per phase (CUDA-graph replay)"),
        "global_streams": streams,
        "streams_per_gpu": streams // max(1, world),
        "ctx": 2048,
        "kv_format": "24-bit split (bf16 high + 8-bit low mantissa)",
        "cache": "inputs larger than L2 (per-GPU KV windows >> 126 MB)",
        "parallelism": f"streams sharded over {world} GPU(s), no hot-path collective",
    }


def boundary_plan(gids: np.ndarray, n_global: int, world: int, n_local: int, every: int, p0: int, chunk: int):
    """Rows that cross a segment boundary before each chunk step.

    Stream g runs its segment clock shifted by phi_g, so boundaries (flush,
    test-time update, next segment) fall at positions p with
    (p + phi_g) % every == 0.  phi spreads the streams evenly over the clock
    and interleaves ranks, so every timed window carries its share of the
    LoRA schedule on every GPU."""
    stride = max(1, every // n_global)
    rank_of = gids // n_local
    j = gids % n_local
    phi = ((j * world + rank_of) * stride) % every
    plan = []
    for t in range(chunk):
        pos = p0 + t
        plan.append([int(i) for i in np.flatnonzero((pos + phi) % every == 0)] if pos > 0 else [])
    return plan


def main():
    args = parse_args()
    rank, world, local = dist_env()
    if args.c2:
        if rank == 0:
            run_c2(args)
        return
    if args.replenish:
        if rank == 0:
            run_replenish(args)
        return
    if args.lora_update:
        if rank == 0:
            run_lora_update(args)
        return
    if args.attention:
        if rank == 0:
            run_attention(args)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.impl == "reference-triton":
        run_reference_triton(args, rank, world)
        return
    import ctypes

    from altxs_b200 import _lib
    from altxs_b200 import codec as C
    from altxs_b200.config import c3_config
    from altxs_b200.engine import DeviceModel, StreamBatch, _stream_handle, words_for_segment
    from altxs_b200.synth import zipf_markov
    from altxs_b200.ttt import LoraTTT

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
        pg = dist
    cfg = c3_config()
    n_local = args.streams // world
    n_global = n_local * world
    W, K = max(3, args.warmup), max(1, args.steps)
    chunk = W + K
    every = cfg.online_retrain_every
    w = C.synth_weights(cfg, seed=WEIGHT_SEED)
    dm = DeviceModel(w, dev, rope_positions=cfg.ctx + chunk + 8, tensor_cores=not args.cuda_cores)
    if args.fusion:
        _lib.check(_lib.lib().altxs_set_step_fusion(4), "altxs_set_step_fusion")
    if args.packed is not None:
        _lib.check(_lib.lib().altxs_set_linear_packed(args.packed), "altxs_set_linear_packed")
    gids = np.arange(rank * n_local, (rank + 1) * n_local)
    data = zipf_markov(cfg.ctx + chunk, cfg.vocab_size, 1000 + gids)  # [n][T]
    symsT = torch.from_numpy(np.ascontiguousarray(data.T)).to(dev)     # [T][n]
    wps = words_for_segment(max(cfg.ctx, chunk), cfg.cdf_bits)
    # each step mode is replayed from a CUDA graph after its first call
    b = StreamBatch(dm, n_local, words_per_stream=wps, hist_len=cfg.ctx + 2, graphs=True)
    ttt = LoraTTT(dm)
    L = _lib.lib()
    stream_h = _stream_handle(dev)

    if args.fill == "prefill":
        # fill every window: code the first ctx symbols (state warm-up, not timed)
        b.encode_chunk(symsT[: cfg.ctx])
    else:
        # seeded random K/V rows (unit-RMS keys, V ~ N(0, 1.5^2)) in the 24-bit
        # split format, every stream positioned with a full window; the symbol
        # ring gets the same seeded symbols
        g = torch.Generator(device=dev)
        g.manual_seed(77 + rank)
        hd = cfg.head_dim
        for li in range(cfg.num_layers):
            for kvi, sd in ((0, 1.0), (1, 1.5)):
                vals = torch.randn((b.n, cfg.num_kv_heads, cfg.ctx, hd), generator=g, device=dev) * sd
                bits = vals.view(torch.int32)
                r = (bits + 0x7F + ((bits >> 8) & 1)) >> 8  # round to 24 bits
                hi = ((r >> 8) & 0xFFFF).to(torch.int32)
                lo = (r & 0xFF).to(torch.uint8)
                hi_bytes = torch.stack(((hi & 0xFF).to(torch.uint8), (hi >> 8).to(torch.uint8)), dim=-1)
                b.kv[:, li, kvi, :, :, : 2 * hd] = hi_bytes.reshape(b.n, cfg.num_kv_heads, cfg.ctx, 2 * hd)
                b.kv[:, li, kvi, :, :, 2 * hd:] = lo
        b.pos.fill_(cfg.ctx - 1)
        b.tok.copy_(symsT[cfg.ctx - 1])
        idx = torch.arange(cfg.ctx, device=dev) % b.hist_len
        b.hist[:, idx] = symsT[: cfg.ctx].T.contiguous()
    torch.cuda.synchronize(dev)
    p0 = cfg.ctx  # symbols coded before the chunk
    plan = boundary_plan(gids, n_global, world, n_local, every, p0, chunk)
    brows = sorted({r for rows in plan for r in rows})
    # snapshot everything the chunk changes, so encode and decode start equal
    pstart = int(b.pos[0].item())
    slots = torch.arange(pstart, pstart + chunk, device=dev) % cfg.ctx
    kv_saved = b.kv.index_select(4, slots)
    tok_saved, pos_saved = b.tok.clone(), b.pos.clone()
    hist_saved = b.hist.clone()
    bidx = torch.as_tensor(brows, dtype=torch.int64, device=dev)
    lora_saved = b.lora.index_select(0, bidx) if brows else None

    def restore():
        b.kv.index_copy_(4, slots, kv_saved)
        b.tok.copy_(tok_saved)
        b.pos.copy_(pos_saved)
        b.hist.copy_(hist_saved)
        if brows:
            b.lora.index_copy_(0, bidx, lora_saved)
            m, v = ttt._moments(b)
            m.index_fill_(0, bidx, 0.0)
            v.index_fill_(0, bidx, 0.0)
        ttt.steps[id(b)] = {}

    # ---- encode the chunk (untimed), segment per boundary -------------------
    chunk_syms = symsT[p0: p0 + chunk]
    segs = [[] for _ in range(b.n)]
    b.ac_init()
    for t in range(chunk):
        rows = plan[t]
        if rows:
            b.ac_flush(rows)
            for r, p in b.segment_bytes(rows).items():
                segs[r].append(p)
            b.ac_init(rows)
            ttt(b, rows, p0 + t)
        b.sym.copy_(chunk_syms[t])
        b.step(_lib.STEP_ENCODE)
    b.ac_flush()
    for r, p in b.segment_bytes(list(range(b.n))).items():
        segs[r].append(p)
    b.check_status()
    bits_total = sum(len(p) for sg in segs for p in sg) * 8
    max_segs = max(len(sg) for sg in segs)
    # host staging of every stream's segments: [n][max_segs][wps] words + bit counts
    stage_h = torch.zeros((b.n, max_segs, wps), dtype=torch.int32)
    nbits_h = torch.zeros((b.n, max_segs), dtype=torch.int64)
    for i, sg in enumerate(segs):
        for k, p in enumerate(sg):
            buf = np.zeros(wps * 4, dtype=np.uint8)
            buf[: len(p)] = np.frombuffer(p, dtype=np.uint8)
            stage_h[i, k] = torch.from_numpy(buf.view(np.int32))
            nbits_h[i, k] = len(p) * 8
    stage_h, nbits_h = stage_h.pin_memory(), nbits_h.pin_memory()
    stage_d = torch.empty_like(stage_h, device=dev)
    nbits_d = torch.empty_like(nbits_h, device=dev)
    seg_idx = torch.zeros(b.n, dtype=torch.int64, device=dev)

    def load_segments(rows, which):
        """bits[rows] <- stage[rows, which]; seed their decoders (device only)."""
        ri = torch.as_tensor(rows, dtype=torch.int64, device=dev)
        wi = torch.as_tensor(which, dtype=torch.int64, device=dev)
        b.bits.index_copy_(0, ri, stage_d[ri, wi])
        nb = nbits_d[ri, wi].contiguous()
        rr = ri.to(torch.int32)
        _lib.check(L.altxs_ac_begin_decode(len(rows), rr.data_ptr(), b.ac.data_ptr(), b.bits.data_ptr(),
                                           nb.data_ptr(), b.words_per_stream, stream_h), "begin_decode")
        return rr, nb  # keep alive until the launch ran

    def decode_chunk(timed_from: int, dsyms: torch.Tensor, on_start=None, on_end=None):
        """Decode the chunk from the restored state; on_start/on_end bracket
        steps [timed_from, chunk)."""
        nxt = [1] * b.n
        keep = [load_segments(list(range(b.n)), [0] * b.n)]
        for t in range(chunk):
            if on_start is not None and t == timed_from:
                on_start()
            rows = plan[t]
            if rows:
                ttt(b, rows, p0 + t)
                keep.append(load_segments(rows, [nxt[r] for r in rows]))
                for r in rows:
                    nxt[r] += 1
            b.step(_lib.STEP_DECODE)
            dsyms[t].copy_(b.sym)
        if on_end is not None:
            on_end()
        return keep

    # ---- device-resident decode: value ------------------------------------
    restore()
    stage_d.copy_(stage_h)
    nbits_d.copy_(nbits_h)
    dsyms = torch.empty((chunk, b.n), dtype=torch.int32, device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    state = {}

    def on_start():  # after the W warm-up steps
        torch.cuda.synchronize(dev)
        if pg:
            pg.barrier()
        torch.cuda.synchronize(dev)
        state["clocks"] = ClockSampler(local)
        time.sleep(0.3)
        state["launches0"] = L.altxs_launch_count()  # eager launches (updates, segment loads)
        state["replays0"] = b.replays
        torch.cuda.nvtx.range_push("timed")
        e0.record()

    def on_end():
        e1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
        per_graph = b.graph_kernels.get((_lib.STEP_DECODE, id(dm.weights_struct)), 0)
        state["launches"] = (L.altxs_launch_count() - state["launches0"]) + (b.replays - state["replays0"]) * per_graph
        state["clk"] = state["clocks"].stop()
        if pg:
            pg.barrier()

    decode_chunk(W, dsyms, on_start, on_end)
    launches, clk = state["launches"], state["clk"]
    ms_local = e0.elapsed_time(e1)
    ms_max = ms_local
    if pg:
        t_ = torch.tensor([ms_local], device=dev)
        pg.all_reduce(t_, op=pg.ReduceOp.MAX)
        ms_max = float(t_.item())
    ncls = len(_lib.KERNEL_CLASSES)
    pms = (ctypes.c_double * ncls)()
    pcnt = (ctypes.c_int64 * ncls)()
    ok = torch.equal(dsyms, chunk_syms)
    b.check_status()
    timed_boundaries = sum(len(plan[t]) for t in range(W, chunk))

    # ---- end to end: host segments in, host symbols out --------------------
    restore()
    out_h = torch.empty((chunk, b.n), dtype=torch.int32).pin_memory()
    dsyms2 = torch.empty((chunk, b.n), dtype=torch.int32, device=dev)
    if pg:
        pg.barrier()
    torch.cuda.synchronize(dev)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    stage_d.copy_(stage_h, non_blocking=True)
    nbits_d.copy_(nbits_h, non_blocking=True)
    decode_chunk(0, dsyms2)
    out_h.copy_(dsyms2, non_blocking=True)
    f1.record()
    torch.cuda.synchronize(dev)
    e2e_ms = f0.elapsed_time(f1)
    if pg:
        t_ = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t_, op=pg.ReduceOp.MAX)
        e2e_ms = float(t_.item())
    ok_e2e = torch.equal(out_h, chunk_syms.cpu())

    # ---- per-class breakdown: the same K steps again, launched one by one
    # (no graph) with every launch bracketed by CUDA events on its stream
    # (event pairs cost time of their own, so this pass is not the value) ---
    b.graphs = False
    restore()
    stage_d.copy_(stage_h)
    nbits_d.copy_(nbits_h)
    dsyms3 = torch.empty((chunk, b.n), dtype=torch.int32, device=dev)

    def on_start_prof():
        torch.cuda.synchronize(dev)
        L.altxs_profile(1)

    def on_end_prof():
        torch.cuda.synchronize(dev)
        L.altxs_profile(0)

    decode_chunk(W, dsyms3, on_start_prof, on_end_prof)
    b.graphs = True
    L.altxs_profile_read(ncls, pms, pcnt)
    breakdown = {name: {"ms_per_step": pms[i] / K, "launches": int(pcnt[i])}
                 for i, name in enumerate(_lib.KERNEL_CLASSES) if pcnt[i]}
    ok = ok and torch.equal(dsyms3, chunk_syms)
    prof = breakdown

    # per-stream (symbols, bytes) gathered over NCCL (the only collective)
    counts = torch.tensor([[chunk, sum(len(p) for p in sg)] for sg in segs], dtype=torch.int64, device=dev)
    if pg:
        allc = [torch.empty_like(counts) for _ in range(world)]
        pg.all_gather(allc, counts)
        counts = torch.cat(allc)
    total_bytes = int(counts[:, 1].sum().item())

    value = n_global * K / (ms_max / 1000.0)
    peaks, peak_kind = load_peaks()
    attn = prof.get("attn_partial")
    roof = None
    if attn:
        # algorithmic bytes of one attention launch (one layer): every KV row of
        # every stream's full window, K and V, 3 bytes per value
        bytes_launch = n_local * cfg.num_kv_heads * cfg.ctx * 2 * 3 * cfg.head_dim
        avg_ms = attn["ms_per_step"] * K / attn["launches"]
        achieved = bytes_launch / (avg_ms / 1000.0) / 1e9
        traffic = None
        tfile = ROOT / "profiles" / "attn_ring_traffic.json"
        if tfile.exists():
            tj = json.loads(tfile.read_text())
            traffic = tj["dram_bytes_per_kv_row"] * n_local * cfg.num_kv_heads * cfg.ctx * 2
        roof = {"bound": "hbm", "kernel": "k_attn_ring", "achieved": achieved,
                "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                "traffic": traffic, "bytes_per_launch": bytes_launch, "avg_launch_ms": avg_ms,
                "peak_source": f"{peak_kind} hbm_gbs",
                "timing": "CUDA events around each attention launch on its stream, over the same K "
                          "steps re-run launch by launch after the graph-replayed timed pass"}
    cpu = same = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the host cores decode some of this GPU's own streams (those without a
        # segment boundary in the chunk: one segment each on both sides), so
        # both bits/symbol figures below describe the same symbols
        crossing = set(brows)
        plain = [int(g) for g in gids if int(g) - rank * n_local not in crossing]
        r = cpu_parallel(args, [1000 + g for g in plain], chunk, args.cpu_seconds)
        cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "bits_per_symbol")}
        done = [s - 1000 - rank * n_local for s in r["stream_bytes"]]
        gpu_bytes = sum(len(p) for i in done for p in segs[i])
        cpu_bytes = sum(r["stream_bytes"].values())
        same = {"streams": len(done), "symbols": len(done) * chunk,
                "gpu": 8.0 * gpu_bytes / (len(done) * chunk), "cpu": 8.0 * cpu_bytes / (len(done) * chunk),
                "delta_pct": 100.0 * (gpu_bytes / cpu_bytes - 1.0),
                "note": "GPU: this engine's fixed-point CDF rule, sliding window; CPU: the "
                        + ("reference's masses and segment-reset context" if r["kind"] == "reference"
                           else "port's CDF rule and sliding window")}
    h2d = int(stage_h.numel() * 4 + nbits_h.numel() * 8)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "sym/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": ms_max / K,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32 math; weights 2/3/4-bit + fp16 scales; KV 24-bit",
        "data": "synthetic: seeded Zipf-Markov streams (alpha 1.1), seeded random mixed-bit weights",
        "config": config_block(world, n_global, args.cuda_cores, args.fusion),
        "bits_per_symbol": bits_total / (n_local * chunk),
        "roundtrip_ok": bool(ok and ok_e2e),
        "ttt_updates_timed": timed_boundaries,
        "roofline": roof,
        "cpu_baseline": cpu,
        "bits_same_symbols": same,
        "e2e": {"value": n_global * chunk / (e2e_ms / 1000.0), "unit": "sym/s",
                "h2d_bytes_per_step": h2d // chunk, "d2h_bytes_per_step": int(b.n * 4),
                "path": "StreamBatch steps + LoraTTT with pinned host segments in, host symbols out"},
        "gpu_launches": int(launches),
        "kernel_ms_per_step": breakdown,
        "clocks": clk,
        "total_payload_bytes": total_bytes,
        "weights_device_bytes": dm.weight_bytes,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
