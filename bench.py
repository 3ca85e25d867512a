#!/usr/bin/env python
"""Benchmark of the NF4 frozen-weight hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload codec] [--impl ours|reference]

Workload ``codec`` (default): one step dequantizes the four
config-2 weight matrices (2048x2048, 4096x4096, 14336x4096, 4096x14336; fp16
~N(0,0.02) with 0.1% x20 outliers, NF4 blocksize 64) to bf16, once from a
plain absmax and once from a double-quantized absmax.  ``value`` is the
whole-job dequant throughput in GB/s of algorithmic bytes (2.5625 B/element
plain, 2.5159 B/element with double quant: packed + absmax read, bf16 written).
Quantize throughput is measured the same way and reported beside it.

With N > 1 (torchrun, one rank per GPU) every rank runs its own replica of
the workload (the codec shards by tensor, no exchange): weak scaling.

Rank 0 prints one JSON line.  Timing: W untimed warm-up steps, then K steps;
each step is bracketed by CUDA events on the launching stream with an L2
flush (a 256 MiB fill) between steps outside the brackets; barrier +
synchronize around the timed region; the max over ranks is reported.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_FLUSH_BYTES = 256 << 20
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


# ----------------------------------------------------------------- helpers --

def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_traffic():
    p = ROOT / "profiles" / "ncu_traffic.json"
    if p.exists():
        return json.loads(p.read_text())
    return {}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.out = None

    def __enter__(self):
        try:
            self.out = open(f"/tmp/stratum_clocks_{os.getpid()}.csv", "w+")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.out, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.out is None:
            return None
        self.out.seek(0)
        rows = [r.split(",") for r in self.out.read().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for nm, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        backend = "nccl" if torch.cuda.is_available() and args.impl == "ours" else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------- codec workload --

DQ_BYTES_PER_ELEM = {False: 0.5 + 4.0 / 64 + 2.0, True: 0.5 + 1.0 / 64 + 4.0 / (64 * 256) + 2.0}
Q_BYTES_PER_ELEM = {False: 2.0 + 0.5 + 4.0 / 64}


class CodecWorkload:
    name = "nf4_codec_config2"

    def __init__(self, device):
        from stratum_b200 import functional as F
        from stratum_b200 import workloads

        self.F = F
        self.device = device
        self.items = []
        for i, shape in enumerate(workloads.CODEC_SHAPES):
            w = workloads.codec_weight(shape, seed=i, device=device)
            packed, st = F.quantize_4bit(w)
            packed_dq, st_dq = F.quantize_4bit(w, compress_statistics=True)
            out = torch.empty(shape, dtype=torch.bfloat16, device=device)
            self.items.append(dict(shape=shape, w=w, n=w.numel(), packed=packed, st=st, packed_dq=packed_dq,
                                   st_dq=st_dq, out=out, qpacked=torch.empty_like(packed),
                                   qabsmax=torch.empty_like(st.absmax)))
        self.n_total = sum(it["n"] for it in self.items)
        self.dequant_bytes = sum(it["n"] * (DQ_BYTES_PER_ELEM[False] + DQ_BYTES_PER_ELEM[True]) for it in self.items)
        self.quant_bytes = sum(it["n"] * Q_BYTES_PER_ELEM[False] for it in self.items)

    def dequant_step(self, events=None):
        """All dequant launches of one step; per-kernel event pairs when ``events`` is a list."""
        F = self.F
        for it in self.items:
            if events is not None:
                e0 = torch.cuda.Event(enable_timing=True)
                e0.record()
            F.dequantize_4bit(it["packed"], it["st"], out=it["out"], out_dtype=torch.bfloat16)
            if events is not None:
                e1 = torch.cuda.Event(enable_timing=True)
                e1.record()
                events.append(("plain", it["n"], e0, e1))
                e0 = torch.cuda.Event(enable_timing=True)
                e0.record()
            F.dequantize_4bit(it["packed_dq"], it["st_dq"], out=it["out"], out_dtype=torch.bfloat16)
            if events is not None:
                e1 = torch.cuda.Event(enable_timing=True)
                e1.record()
                events.append(("dq", it["n"], e0, e1))

    def quant_step(self):
        from stratum_b200 import _lib, codebook

        L = _lib.lib()
        st = _lib.stream_of(self.device)
        thr = codebook.nf4_thresholds(self.device)
        for it in self.items:
            _lib.check(L.stratum_nf4_quantize(_lib.ptr(it["w"]), 1, it["n"], 64, _lib.ptr(thr), _lib.ptr(it["qpacked"]),
                                              _lib.ptr(it["qabsmax"]), st), "quantize")


def run_codec(args, world, rank, local):
    from stratum_b200 import _lib

    dev = torch.device("cuda", torch.cuda.current_device())
    wl = CodecWorkload(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)

    for _ in range(args.warmup):
        wl.dequant_step()
        wl.quant_step()
    torch.cuda.synchronize()

    # --- timed region: K dequant steps (value) -------------------------------
    step_ms, kern = [], []
    barrier(world)
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    t_wall = time.perf_counter()
    with ClockSampler(dev.index) as clocks:
        for _ in range(args.steps):
            flush.fill_(1)  # L2 flush between timed steps (outside the event brackets)
            ev = []
            wl.dequant_step(ev)
            kern.append(ev)
        torch.cuda.synchronize()
        t_wall = time.perf_counter() - t_wall
        launches = _lib.launch_count() - launches0
        barrier(world)
        for ev in kern:
            step_ms.append(sum(e0.elapsed_time(e1) for _, _, e0, e1 in ev))
        # quantize, timed the same way
        q_ms = []
        for _ in range(args.steps):
            flush.fill_(1)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            wl.quant_step()
            e1.record()
            q_ms.append((e0, e1))
        torch.cuda.synchronize()
    q_ms = [a.elapsed_time(b) for a, b in q_ms]
    ms = max_over_ranks(statistics.mean(step_ms), world)
    qms = max_over_ranks(statistics.mean(q_ms), world)
    value = wl.dequant_bytes * world / (ms * 1e-3) / 1e9
    qvalue = wl.quant_bytes * world / (qms * 1e-3) / 1e9

    # dominant kernel: plain dequant to bf16 (k_dequant<bf16,false>)
    plain = [(n, e0.elapsed_time(e1)) for ev in kern for kind, n, e0, e1 in ev if kind == "plain"]
    plain_bytes = sum(n * DQ_BYTES_PER_ELEM[False] for n, _ in plain)
    plain_ms = sum(t for _, t in plain)
    achieved = plain_bytes / (plain_ms * 1e-3) / 1e9
    peaks = load_peaks()
    traffic_tab = load_traffic().get("k_dequant_bf16", {})
    per_launch_elems = plain_bytes / DQ_BYTES_PER_ELEM[False] / len(plain)
    traffic = traffic_tab.get("bytes_per_elem")
    roofline = {
        "bound": "hbm",
        "kernel": "k_dequant<bf16,plain>",
        "achieved": round(achieved, 1),
        "peak": peaks["hbm_gbs"],
        "unit": "GB/s",
        "frac": round(achieved / peaks["hbm_gbs"], 4),
        "frac_of": peaks["source"],
        "frac_nominal_8000": round(achieved / NOMINAL_HBM_GBS, 4),
        "algorithmic_bytes_per_launch": round(plain_bytes / len(plain)),
        "traffic": None if traffic is None else round(traffic * per_launch_elems),
        "traffic_source": traffic_tab.get("source"),
    }

    e2e = run_codec_e2e(args, wl, world) if rank == 0 or world > 1 else None
    cpu = run_cpu_baseline_codec() if (world == 1 and rank == 0 and not args.no_cpu_baseline) else None
    clk = clocks.summary()
    return {
        "metric": "nf4_dequant_GBps",
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8->bf16",
        "data": "synthetic: seeded fp16 ~N(0,0.02) with 0.1% x20 outliers, NF4 blocksize 64 (BASELINE config 2)",
        "config": {"workload": "codec: dequant of 2048^2, 4096^2, 14336x4096, 4096x14336 to bf16, plain and "
                               "double-quant absmax", "elements_per_step": wl.n_total, "blocksize": 64,
                   "parallelism": f"replicas x{world}", "l2": "256 MiB fill between timed steps (outside events)"},
        "quantize": {"value": round(qvalue, 1), "unit": "GB/s", "ms_per_step": round(qms, 4),
                     "frac": round(qvalue / peaks["hbm_gbs"], 4)},
        "roofline": roofline,
        "e2e": e2e,
        "cpu_baseline": cpu,
        "gpu_launches": int(launches),
        "wall_s_timed": round(t_wall, 4),
        "clocks": clk,
    }


def run_codec_e2e(args, wl, world):
    """Same metric through the reference-facing call with host buffers.

    Each step: pinned-host -> device copy of every matrix's NF4 payload
    (packed + absmax), ``dequantize_4bit`` to bf16 on the device, and a
    device -> host read of a 4 KiB slice of each result.
    """
    F = wl.F
    host = []
    for it in wl.items:
        host.append((it["packed"].cpu().pin_memory(), it["st"].absmax.cpu().pin_memory()))
    readback = torch.empty(len(wl.items) * 2048, dtype=torch.bfloat16).pin_memory()
    h2d = sum(p.numel() + a.numel() * 4 for p, a in host)
    d2h = readback.numel() * 2
    from stratum_b200.functional import QuantState

    def step():
        for i, (it, (p, a)) in enumerate(zip(wl.items, host)):
            pd = p.to(wl.device, non_blocking=True)
            ad = a.to(wl.device, non_blocking=True)
            st = QuantState(ad, it["st"].shape, it["st"].code, 64, "nf4", it["st"].dtype)
            out = F.dequantize_4bit(pd, st, out_dtype=torch.bfloat16)
            readback[i * 2048:(i + 1) * 2048].copy_(out.view(-1)[-2048:], non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(max(1, args.warmup)):
        step()
    barrier(world)
    t = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t) / args.steps
    dt = max_over_ranks(dt, world)
    plain_bytes = sum(it["n"] * DQ_BYTES_PER_ELEM[False] for it in wl.items)
    return {"value": round(plain_bytes * world / dt / 1e9, 2), "unit": "GB/s", "ms_per_step": round(dt * 1e3, 3),
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "path": "functional.dequantize_4bit (plain absmax) with pinned host payloads"}


def run_cpu_baseline_codec(budget_s: float = 12.0):
    """The C restatement of the codec timed on all host cores on a bounded sample."""
    import numpy as np

    from oracle import nf4_oracle_c
    from stratum_b200 import workloads

    oc = nf4_oracle_c.load()
    w = workloads.codec_weight((4096, 4096), seed=1, device="cpu")
    packed, absmax = oc.quantize(w, 64)
    n = w.numel()
    oc.dequantize(packed, absmax, n, 64, "bfloat16")  # warm
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        oc.dequantize(packed, absmax, n, 64, "bfloat16")
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    del np
    return {"value": round(n * DQ_BYTES_PER_ELEM[False] / dt / 1e9, 3), "unit": "GB/s", "cores": oc.threads,
            "kind": "port", "sample": f"oracle C dequant of a 4096x4096 NF4 matrix to bf16, {reps} reps in "
                                      f"{budget_s:.0f} s, {oc.threads} OpenMP threads",
            "cpu": _cpu_model()}


def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


# --------------------------------------------------------- reference arm --

def run_reference(args, world, rank):
    """The reference's CPU implementation of the path, timed on the host cores.

    The reference's NF4 arithmetic lives in bitsandbytes, which is absent here
    and cannot be installed offline, so its restatement (oracle/, C + OpenMP)
    stands in ("port").  Same workload, metric and unit as our arm.
    """
    if rank != 0:
        return None
    import numpy as np

    from oracle import nf4_oracle_c
    from stratum_b200 import workloads

    oc = nf4_oracle_c.load()
    items = []
    for i, shape in enumerate(workloads.CODEC_SHAPES):
        w = workloads.codec_weight(shape, seed=i, device="cpu")
        packed, absmax = oc.quantize(w, 64)
        q, a2, c2, off = oc.quantize_absmax_dq(absmax)
        items.append((w.numel(), packed, absmax, q, a2, c2, off))

    def step():
        for n, packed, absmax, q, a2, c2, off in items:
            oc.dequantize(packed, absmax, n, 64, "bfloat16")
            oc.dequantize_dq(packed, q, a2, c2, off, n, 64, "bfloat16")

    for _ in range(args.warmup):
        step()
    t = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t) / args.steps
    total = sum(n * (DQ_BYTES_PER_ELEM[False] + DQ_BYTES_PER_ELEM[True]) for n, *_ in items)
    value = total / dt / 1e9
    del np
    return {
        "impl": "reference",
        "metric": "nf4_dequant_GBps",
        "value": round(value, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8->bf16",
        "data": "synthetic: seeded fp16 ~N(0,0.02) with 0.1% x20 outliers, NF4 blocksize 64 (BASELINE config 2)",
        "config": {"workload": "codec: dequant of 2048^2, 4096^2, 14336x4096, 4096x14336 to bf16, plain and "
                               "double-quant absmax", "blocksize": 64, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": oc.threads, "kind": "port",
                         "sample": "full config-2 workload per step (bitsandbytes absent: oracle C restatement)",
                         "cpu": _cpu_model()},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# -------------------------------------------------------------------- main --

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("codec",), default="codec")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            out = run_reference(args, world, rank)
        else:
            if not torch.cuda.is_available():
                raise SystemExit("bench.py: no CUDA device (the product path has no CPU fallback)")
            out = run_codec(args, world, rank, local)
        if rank == 0 and out is not None:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
