#!/usr/bin/env python3
"""Throughput benchmark: Kokoro decoder + generator (rokoko's hot path) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: decoder/generator only, FP32 semantics, synthetic
features asr [400, 512] ~ N(0,1), F0 [800] = 200 Hz +-50 Hz seeded walk,
N [800] ~ N(0, 0.1), style [128] ~ N(0, 0.1), random-init weights in the KOKO
v1 layout -> 240,000 samples = 10.0 s of 24 kHz audio per utterance.  A step is
one utterance per GPU (independent utterances on every rank, no collective;
weak scaling).  Metric: audio-seconds per second over all GPUs.

`value` is timed on the device with CUDA events on the library's stream,
inputs resident in HBM; L2 is flushed (256 MB write) before every timed step,
outside the events.  `e2e` is the same metric through the host-buffer C-ABI
call rk_decode_features (pinned host inputs, host PCM out) timed with the
wall clock.  `roofline` is the tcgen05 conv kernel measured live on a second
pass of the same steps, replayed as a profiling CUDA graph with every lane on
one stream, each conv launch bracketed by its own event nodes (the kernels'
own time).  Under torchrun each rank
drives LOCAL_RANK's GPU; ranks meet at a barrier and the max over ranks is
reported by rank 0.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L_FRAMES = 400
AUDIO_S = 600 * L_FRAMES / 24000.0  # 10.0 s per utterance
METRIC = "audio-sec/sec (RTF^-1)"
UNIT = "audio-s/s"
WORKLOAD = "config1: decoder+generator, L=400 frames -> 10.0 s of 24 kHz audio per utterance per GPU, FP32"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="clk", suffix=".csv")
        os.close(fd)
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.out, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) < 9:
                    continue
                try:
                    sm.append(float(p[1]))
                    mx = max(mx, float(p[2]))
                except ValueError:
                    continue
                for nm, v in zip(names, p[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(nm)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU legs
def cpu_oracle_throughput(blob, L: int, runs: int):
    """Oracle (CPU restatement) decode of `runs` utterances of L frames, all host threads."""
    import oracle
    from rokoko_b200 import configs
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    oracle.set_threads(threads)
    m = oracle.Oracle(blob)
    c = configs.config1(seed=7, L=L)
    t0 = time.perf_counter()
    for _ in range(runs):
        m.decode_features(c.asr, c.f0, c.n, c.style)
    dt = time.perf_counter() - t0
    m.close()
    return runs * 600 * L / 24000.0 / dt, threads, dt


def run_reference(args, world, rank):
    """`--impl reference`: the CPU restatement of the reference's decoder path
    (the reference's own CPU backend is absent from its tree), timed on this
    box's host cores; rank 0 only."""
    if rank != 0:
        return
    from rokoko_b200 import koko
    blob = koko.random_v1_blob(0)
    L = 100  # bounded per-step sample: 2.5 s of audio
    for _ in range(args.warmup):
        cpu_oracle_throughput(blob, L, 1)
    v, threads, dt = cpu_oracle_throughput(blob, L, args.steps)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * dt / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": f"L={L} frames (2.5 s audio) per step",
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{args.steps} decodes of L={L} frames (CPU FP32 restatement; the reference "
                                   "ships no CPU backend)"},
        "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU leg
def run_ours(args, world, rank, local):
    import numpy as np
    import torch
    import torch.distributed as dist
    from rokoko_b200 import configs, koko
    from rokoko_b200.context import FP32, RK_PROFILE_CONV, RK_PROFILE_SERIAL, Context

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    blob = koko.random_v1_blob(0)
    ctx = Context(local, FP32)
    ctx.load_weights(blob)
    c = configs.config1(seed=rank, L=L_FRAMES)
    d_asr = torch.from_numpy(c.asr).to(dev)
    d_f0 = torch.from_numpy(c.f0).to(dev)
    d_n = torch.from_numpy(c.n).to(dev)
    d_st = torch.from_numpy(c.style).to(dev)
    d_pcm = torch.empty(600 * L_FRAMES, dtype=torch.float32, device=dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MB > 126 MB L2
    ext = torch.cuda.ExternalStream(ctx.stream, device=dev)

    def step():
        ctx.decode_features_device(d_asr.data_ptr(), d_f0.data_ptr(), d_n.data_ptr(), d_st.data_ptr(), L_FRAMES,
                                   d_pcm.data_ptr())

    torch.cuda.synchronize(dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    clocks = ClockSampler(local)

    # ---- timed region: graph replays, device events around every step
    k0 = ctx.kernel_count()
    barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    with torch.cuda.stream(ext):
        for k in range(args.steps):
            flush.zero_()
            ev0[k].record(ext)
            step()
            ev1[k].record(ext)
    torch.cuda.synchronize(dev)
    barrier()
    clk = clocks.stop()
    launches = ctx.kernel_count() - k0
    t_ms = sum(a.elapsed_time(b) for a, b in zip(ev0, ev1))
    t_ms = max_over_ranks(t_ms)
    value = world * AUDIO_S * args.steps / (t_ms / 1000.0)

    # ---- conv roofline: the same K steps again as a profiling graph with every lane on
    # the context stream (RK_PROFILE_CONV | RK_PROFILE_SERIAL), so each conv launch is
    # bracketed by its own pair of event nodes and runs alone on the GPU; the graph's
    # total device time gives the conv share of a serialised decode
    ctx.profile(RK_PROFILE_CONV | RK_PROFILE_SERIAL)
    step()
    ctx.profile_read()
    ctx.profile(RK_PROFILE_CONV | RK_PROFILE_SERIAL)
    torch.cuda.synchronize(dev)
    serial_ms = 0.0
    ps0, ps1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(ext):
        for k in range(args.steps):
            flush.zero_()
            ps0.record(ext)
            step()
            ps1.record(ext)
            ctx.profile_read()  # synchronises; the next replay re-records the same event nodes
            serial_ms += ps0.elapsed_time(ps1)
    conv_ms, conv_flops, conv_n = ctx.profile_read()
    ctx.profile(False)

    # ---- end to end through the host-buffer API (pinned inputs, host PCM)
    h_asr = torch.from_numpy(c.asr).pin_memory().numpy()
    h_f0 = torch.from_numpy(c.f0).pin_memory().numpy()
    h_n = torch.from_numpy(c.n).pin_memory().numpy()
    h_st = torch.from_numpy(c.style).pin_memory().numpy()
    for _ in range(2):
        ctx.decode_features(h_asr, h_f0, h_n, h_st)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        pcm = ctx.decode_features(h_asr, h_f0, h_n, h_st)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    e2e = world * AUDIO_S * args.steps / e2e_s
    h2d = c.asr.nbytes + c.f0.nbytes + c.n.nbytes + c.style.nbytes
    d2h = pcm.nbytes

    if rank == 0:
        peaks, src = measured_peaks()
        peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
        achieved = conv_flops / (conv_ms * 1e-3) / 1e12 if conv_ms > 0 else 0.0
        traffic = None
        tp = os.path.join(ROOT, "profiles", "conv_tc_traffic.json")
        if os.path.exists(tp):
            with open(tp) as f:
                traffic = json.load(f).get("dram_bytes_per_launch")
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            v, threads, dt = cpu_oracle_throughput(blob, L_FRAMES, 2)
            cpu = {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": f"2 decodes of the config-1 utterance (L={L_FRAMES}, 20 s of audio, {dt:.1f} s of "
                             "CPU work) with the CPU FP32 restatement; the reference ships no CPU backend"}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {
                "workload": WORKLOAD, "L": L_FRAMES, "audio_s_per_step_per_gpu": AUDIO_S,
                "precision": "FP32 semantics: 3-pass split-bf16 tcgen05 products, FP32 accumulate",
                "parallelism": f"dp{world} (independent utterances per GPU, no collective)",
                "l2": "256 MB L2 flush before every timed step (outside the events); per-step working set > L2",
                "launches_per_step": launches / args.steps,
            },
            "clocks": clk,
            "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "roofline": {
                "kernel": "conv_tc_kernel (tcgen05 implicit-GEMM Conv1d / ConvTranspose1d)",
                "bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "peak_source": f"bf16_tflops_sustained of {src}",
                "flops": "algorithmic 2*C_in*C_out*K*T_out per conv (x T_in for ConvTranspose1d); the FP32 "
                         "semantics issue 3 bf16 products per algorithmic product",
                "issued_frac": round(3 * achieved / peak, 4),
                "conv_launches": conv_n, "conv_ms_per_step": round(conv_ms / args.steps, 4),
                "serial_step_ms": round(serial_ms / args.steps, 4),
                "conv_share_of_serial_step": round(conv_ms / serial_ms, 4) if serial_ms > 0 else None,
                "step_ms": round(t_ms / args.steps, 4),
                "measured": "second pass of the same K steps as a CUDA graph with all lanes on one stream; each conv "
                            "launch bracketed by its own event nodes (kernel time alone on the GPU); issued_frac counts "
                            "the 3 bf16 products per algorithmic product of the FP32 semantics",
            },
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse_args()
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
