#!/usr/bin/env python
"""Benchmark: decode symbols/sec of the 33M, 3.15-bpw model-and-code loop.

Workload (BASELINE config "box-scale sharded run"): 2048 independent streams
split evenly over N GPUs (one process per GPU), the 33M model (8L/512d/8h,
MLP 2048, V 16384) with seeded random mixed 2/3/4-bit weights, sliding
window filled to 2048 of 2048, symbols from the seeded Zipf-Markov source.
A step decodes one symbol for every stream on every GPU: model step over the
full window, logits -> integer CDF, range decode.  Streams share no data, so
there is no collective on the hot path (weak per-stream work, fixed total
streams -> "strong" scaling); NCCL only gathers per-stream byte counts.

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
cuda synchronize, CUDA events on the launch stream, max over ranks.  The KV
windows (~103 GB per GPU at N=1) are far larger than L2, so every step
streams its inputs from HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""

from __future__ import annotations

import argparse
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
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--streams", type=int, default=GLOBAL_STREAMS, help="global stream count")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--fill", choices=("prefill", "random"), default="prefill",
                    help="how the windows are filled before timing: code the preceding 2048 symbols "
                         "(default) or write seeded random K/V rows (profiling runs: same per-step work, "
                         "no 2048-step warm-up)")
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


def run_reference(args, rank, world):
    """CPU reference arm: the reference's eager decode path (oracle port)."""
    if rank != 0:
        return
    from altxs_b200 import codec as C
    from altxs_b200.config import c3_config
    from oracle.baseline import cpu_decode_baseline

    cfg = c3_config()
    w = C.synth_weights(cfg, seed=WEIGHT_SEED)
    per_step = []
    for _ in range(max(1, args.warmup)):
        cpu_decode_baseline(w, target_s=min(2.0, args.cpu_seconds), seed=1)
    t0 = time.perf_counter()
    res = None
    for k in range(max(1, min(args.steps, 3))):
        res = cpu_decode_baseline(w, target_s=args.cpu_seconds, seed=1 + k)
        per_step.append(res["value"])
    value = float(statistics.median(per_step))
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "sym/s",
        "n_gpus": world,
        "steps": len(per_step),
        "warmup": args.warmup,
        "ms_per_step": 1000.0 / value,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic Zipf-Markov (alpha 1.1), seeded random mixed-bit weights",
        "config": config_block(world, GLOBAL_STREAMS),
        "cpu_baseline": {"value": value, "unit": "sym/s", "cores": res["cores"], "kind": res["kind"],
                         "sample": res["sample"]},
        "e2e": {"value": value, "unit": "sym/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "bits_per_symbol": res["bits_per_symbol"],
        "wall_s": time.perf_counter() - t0,
    }
    print(json.dumps(line), flush=True)


def config_block(world: int, streams: int) -> dict:
    return {
        "workload": "box-scale sharded decode: 2048 independent streams split over N GPUs, 33M model "
                    "(8L/512d/8h, MLP 2048, V 16384) at mixed 2/3/4-bit 3.15 bpw, ctx 2048 window full",
        "global_streams": streams,
        "streams_per_gpu": streams // max(1, world),
        "ctx": 2048,
        "kv_format": "24-bit split (bf16 high + 8-bit low mantissa)",
        "cache": "inputs larger than L2 (per-GPU KV windows >> 126 MB)",
        "parallelism": f"streams sharded over {world} GPU(s), no hot-path collective",
    }


def main():
    args = parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    from altxs_b200 import _lib
    from altxs_b200 import codec as C
    from altxs_b200.config import c3_config
    from altxs_b200.engine import DeviceModel, StreamBatch, words_for_segment
    from altxs_b200.synth import zipf_markov

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
        pg = dist
    cfg = c3_config()
    cfg.retrain_mode = "lora"  # adapters present in every step (B = 0 before the first boundary)
    n_local = args.streams // world
    W, K = max(3, args.warmup), max(1, args.steps)
    chunk = W + K
    w = C.synth_weights(cfg, seed=WEIGHT_SEED)
    dm = DeviceModel(w, dev, rope_positions=cfg.ctx + chunk + 8)
    gids = np.arange(rank * n_local, (rank + 1) * n_local)
    data = zipf_markov(cfg.ctx + chunk, cfg.vocab_size, 1000 + gids)  # [n][T]
    symsT = torch.from_numpy(np.ascontiguousarray(data.T)).to(dev)     # [T][n]
    b = StreamBatch(dm, n_local, words_per_stream=words_for_segment(max(cfg.ctx, chunk), cfg.cdf_bits))
    L = _lib.lib()

    if args.fill == "prefill":
        # fill every window: code the first ctx symbols (state warm-up, not timed)
        b.encode_chunk(symsT[: cfg.ctx])
    else:
        # seeded random K/V rows (unit-RMS keys, V ~ N(0, 1.5^2)) in the 24-bit
        # split format, every stream positioned with a full window
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
    torch.cuda.synchronize(dev)
    # snapshot what the timed chunk overwrites, so encode and decode start equal
    p0 = int(b.pos[0].item())
    slots = torch.arange(p0, p0 + chunk, device=dev) % cfg.ctx
    kv_saved = b.kv.index_select(4, slots)
    tok_saved, pos_saved = b.tok.clone(), b.pos.clone()

    def restore():
        b.kv.index_copy_(4, slots, kv_saved)
        b.tok.copy_(tok_saved)
        b.pos.copy_(pos_saved)

    chunk_syms = symsT[cfg.ctx: cfg.ctx + chunk]
    payloads = b.encode_chunk(chunk_syms)
    bits_total = sum(len(p) for p in payloads) * 8
    words_h, nbits_h = b.pack_payloads(payloads)

    # ---- device-resident decode: value ------------------------------------
    restore()
    b.bits.copy_(words_h.to(dev))
    nb_d = nbits_h.to(dev)
    _lib.check(L.altxs_ac_begin_decode(b.n, None, b.ac.data_ptr(), b.bits.data_ptr(), nb_d.data_ptr(),
                                       b.words_per_stream, torch.cuda.current_stream(dev).cuda_stream), "bd")
    dsyms = torch.empty((chunk, b.n), dtype=torch.int32, device=dev)
    for t in range(W):
        b.step(_lib.STEP_DECODE)
        dsyms[t].copy_(b.sym)
    if pg:
        pg.barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    time.sleep(0.3)
    L.altxs_profile(1)
    launches0 = L.altxs_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    e0.record()
    for t in range(W, chunk):
        b.step(_lib.STEP_DECODE)
        dsyms[t].copy_(b.sym)
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    launches = L.altxs_launch_count() - launches0
    L.altxs_profile(0)
    clk = clocks.stop()
    if pg:
        pg.barrier()
    ms_local = e0.elapsed_time(e1)
    ms_max = ms_local
    if pg:
        t = torch.tensor([ms_local], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms_max = float(t.item())
    import ctypes

    ncls = len(_lib.KERNEL_CLASSES)
    pms = (ctypes.c_double * ncls)()
    pcnt = (ctypes.c_int64 * ncls)()
    L.altxs_profile_read(ncls, pms, pcnt)
    prof = {name: {"ms_per_step": pms[i] / K, "launches": int(pcnt[i])}
            for i, name in enumerate(_lib.KERNEL_CLASSES) if pcnt[i]}
    ok = torch.equal(dsyms, chunk_syms)
    b.check_status()

    # ---- end to end through the chunk API, host buffers --------------------
    restore()
    out_h = torch.empty((chunk, b.n), dtype=torch.int32).pin_memory()
    if pg:
        pg.barrier()
    torch.cuda.synchronize(dev)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    b.decode_chunk(words_h, nbits_h, chunk, out=out_h)
    f1.record()
    torch.cuda.synchronize(dev)
    e2e_ms = f0.elapsed_time(f1)
    if pg:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    ok_e2e = torch.equal(out_h, chunk_syms.cpu())

    # per-stream (symbols, bytes) gathered over NCCL (the only collective)
    counts = torch.tensor([[chunk, len(p)] for p in payloads], dtype=torch.int64, device=dev)
    if pg:
        allc = [torch.empty_like(counts) for _ in range(world)]
        pg.all_gather(allc, counts)
        counts = torch.cat(allc)
    total_bytes = int(counts[:, 1].sum().item())
    n_global = n_local * world

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
        tfile = ROOT / "profiles" / "attn_partial_traffic.json"
        if tfile.exists():
            tj = json.loads(tfile.read_text())
            traffic = tj["dram_bytes_per_kv_row"] * n_local * cfg.num_kv_heads * cfg.ctx * 2
        roof = {"bound": "hbm", "kernel": "k_attn_partial", "achieved": achieved,
                "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                "traffic": traffic, "bytes_per_launch": bytes_launch, "avg_launch_ms": avg_ms,
                "peak_source": f"{peak_kind} hbm_gbs"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.baseline import cpu_decode_baseline

        r = cpu_decode_baseline(w, target_s=args.cpu_seconds, seed=1)
        cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
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
        "config": config_block(world, n_global),
        "bits_per_symbol": bits_total / (n_local * chunk),
        "roundtrip_ok": bool(ok and ok_e2e),
        "roofline": roof,
        "cpu_baseline": cpu,
        "e2e": {"value": n_global * chunk / (e2e_ms / 1000.0), "unit": "sym/s",
                "h2d_bytes_per_step": int(words_h.numel() * 4 + nbits_h.numel() * 8) // chunk,
                "d2h_bytes_per_step": int(b.n * 4),
                "path": "StreamBatch.decode_chunk (pinned host segment in, host symbols out)"},
        "gpu_launches": int(launches),
        "kernel_ms_per_step": prof,
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
