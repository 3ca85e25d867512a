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
    """SM clocks and throttle reasons sampled every 5 ms (NVML, in a thread) during the timed region."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, gpu_index: int, period_s: float = 0.005):
        self.gpu_index = gpu_index
        self.period = period_s
        self.samples = []
        self.max_mhz = None
        self._stop = None
        self._thread = None
        self._nvml = None

    def __enter__(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            # NVML enumerates all GPUs; map the CUDA index through the PCI address
            h = None
            try:
                pr = torch.cuda.get_device_properties(self.gpu_index)
                addr = f"{int(pr.pci_domain_id):08X}:{int(pr.pci_bus_id):02X}:{int(pr.pci_device_id):02X}.0"
                h = pynvml.nvmlDeviceGetHandleByPciBusId(addr.encode())
            except Exception:
                h = None
            if h is None:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[self.gpu_index]) if vis and vis.split(",")[0].isdigit() else self.gpu_index
                h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self._h = h
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None
            return self
        self._stop = threading.Event()

        def loop():
            nv = self._nvml
            while not self._stop.is_set():
                try:
                    mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                    self.samples.append((mhz, rs))
                except Exception:
                    pass
                self._stop.wait(self.period)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return None
        mhz = [m for m, _ in self.samples]
        reasons = sorted({name for _, rs in self.samples for name, bit in self.REASONS.items() if rs & bit})
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(mhz), "source": "nvml"}


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
        """All dequant launches of one step: the four matrices with plain absmax in one
        batched launch (``functional.dequantize_4bit_many``, what ``ensure_weights`` does
        per layer), then the four with double-quant absmax in another.  ``events``: list
        collecting (kind, n, e0, e1) external-event pairs around every launch (recorded as
        graph nodes when captured)."""
        F = self.F
        for kind, pk, stk in (("plain", "packed", "st"), ("dq", "packed_dq", "st_dq")):
            if events is not None:
                e0 = torch.cuda.Event(enable_timing=True, external=True)
                e1 = torch.cuda.Event(enable_timing=True, external=True)
                e0.record()
            F.dequantize_4bit_many([(it[pk], it[stk], it["out"]) for it in self.items], out_dtype=torch.bfloat16)
            if events is not None:
                e1.record()
                events.append((kind, self.n_total, e0, e1))

    def quant_step(self):
        from stratum_b200 import _lib, codebook

        L = _lib.lib()
        st = _lib.stream_of(self.device)
        thr = codebook.nf4_thresholds(self.device)
        for it in self.items:
            _lib.check(L.stratum_nf4_quantize(_lib.ptr(it["w"]), 1, it["n"], 64, _lib.ptr(thr), _lib.ptr(it["qpacked"]),
                                              _lib.ptr(it["qabsmax"]), st), "quantize")


def capture(fn):
    """Capture ``fn()`` into a CUDA graph (after one eager warm-up call); returns (graph, result, launches)."""
    from stratum_b200 import _lib

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    n0 = _lib.launch_count()
    with torch.cuda.graph(g):
        res = fn()
    return g, res, _lib.launch_count() - n0


def run_codec(args, world, rank, local):
    dev = torch.device("cuda", torch.cuda.current_device())
    wl = CodecWorkload(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)

    # one step = one replay of a CUDA graph holding the step's launches (the
    # kernels are a few microseconds each; eager Python dispatch would starve the GPU)
    ev = []
    g_dq, _, dq_launches = capture(lambda: (ev.clear(), wl.dequant_step(ev)))
    g_q, _, q_launches = capture(wl.quant_step)

    for _ in range(args.warmup):
        g_dq.replay()
        g_q.replay()
    torch.cuda.synchronize()

    step_ms, plain = [], []
    barrier(world)
    torch.cuda.synchronize()
    t_wall = time.perf_counter()
    with ClockSampler(dev.index) as clocks:
        for _ in range(args.steps):
            flush.fill_(1)  # L2 flush between timed steps (outside the event brackets)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            g_dq.replay()
            e1.record()
            e1.synchronize()
            step_ms.append(e0.elapsed_time(e1))
            plain += [(n, a.elapsed_time(b)) for kind, n, a, b in ev if kind == "plain"]
        torch.cuda.synchronize()
        t_wall = time.perf_counter() - t_wall
        barrier(world)
        q_ms = []
        for _ in range(args.steps):
            flush.fill_(1)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            g_q.replay()
            e1.record()
            e1.synchronize()
            q_ms.append(e0.elapsed_time(e1))
    ms = max_over_ranks(statistics.mean(step_ms), world)
    qms = max_over_ranks(statistics.mean(q_ms), world)
    value = wl.dequant_bytes * world / (ms * 1e-3) / 1e9
    qvalue = wl.quant_bytes * world / (qms * 1e-3) / 1e9

    # dominant kernel: plain dequant to bf16 of all four matrices (k_dequant_many<bf16, plain absmax>)
    plain_bytes = sum(n * DQ_BYTES_PER_ELEM[False] for n, _ in plain)
    plain_ms = sum(t for _, t in plain)
    achieved = plain_bytes / (plain_ms * 1e-3) / 1e9
    big = [(n, t) for n, t in plain if n == max(nn for nn, _ in plain)]
    big_gbs = sum(n * DQ_BYTES_PER_ELEM[False] for n, _ in big) / (sum(t for _, t in big) * 1e-3) / 1e9
    peaks = load_peaks()
    traffic_tab = load_traffic().get("k_dequant_many_bf16", {})
    per_launch_elems = plain_bytes / DQ_BYTES_PER_ELEM[False] / len(plain)
    traffic = traffic_tab.get("bytes_per_elem")
    roofline = {
        "bound": "hbm",
        "kernel": "k_dequant_many<bf16, plain absmax> (the four config-2 matrices in one launch)",
        "achieved": round(achieved, 1),
        "peak": peaks["hbm_gbs"],
        "unit": "GB/s",
        "frac": round(achieved / peaks["hbm_gbs"], 4),
        "frac_of": peaks["source"],
        "frac_nominal_8000": round(achieved / NOMINAL_HBM_GBS, 4),
        "largest_launch_GBps": round(big_gbs, 1),
        "algorithmic_bytes_per_launch": round(plain_bytes / len(plain)),
        "traffic": None if traffic is None else round(traffic * per_launch_elems),
        "traffic_source": traffic_tab.get("source"),
    }

    e2e = run_codec_e2e(args, wl, world)
    cpu = run_cpu_baseline_codec() if (world == 1 and rank == 0 and not args.no_cpu_baseline) else None
    clk = clocks.summary()
    n_total = wl.n_total
    del wl, g_dq, g_q
    torch.cuda.empty_cache()
    lin = None if args.no_linear else run_linear_metrics(args, world, flush)
    if lin is not None:
        lin["sweep_fused_vs_dequant_cublas"] = run_linear_sweep(flush)
    moe = None if args.no_experts else run_experts_metrics(args, world, flush)
    del flush
    torch.cuda.empty_cache()
    pipe = None if args.no_pipeline else run_pipeline_metrics(args, world, rank, local)
    # configs 3 and 4 as their own sections: Qwen3-0.6B on one GPU (CUDA-graph microbatches),
    # the Qwen3-30B-A3B-shaped MoE (router aux loss on) over every N of the run
    pipe3 = pipe4 = None
    if not args.no_pipeline and not args.no_pipeline_configs:
        if world == 1:
            pipe3 = run_pipeline_metrics(args, world, rank, local, model="qwen3-0.6b")
        pipe4 = run_pipeline_metrics(args, world, rank, local, model="qwen3-30b-a3b")
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
                               "double-quant absmax (one CUDA-graph replay per step)", "elements_per_step": n_total,
                   "blocksize": 64, "parallelism": f"replicas x{world}",
                   "l2": "256 MiB fill between timed steps (outside events)"},
        "quantize": {"value": round(qvalue, 1), "unit": "GB/s", "ms_per_step": round(qms, 4),
                     "frac": round(qvalue / peaks["hbm_gbs"], 4)},
        "roofline": roofline,
        "e2e": e2e,
        "cpu_baseline": cpu,
        "gpu_launches": int(dq_launches) * args.steps,
        "wall_s_timed": round(t_wall, 4),
        "clocks": clk,
        "nf4_linear": lin,
        "nf4_moe_experts": moe,
        "pipeline": pipe,
        "pipeline_qwen3_0_6b": pipe3,
        "pipeline_qwen3_30b_a3b": pipe4,
    }


# ---------------------------------------------------------- linear workload --

LINEAR_SHAPES = ((14336, 4096), (4096, 14336))  # [N, K]: up/gate-proj and down-proj of Llama-3-8B
LINEAR_T = 8192
LINEAR_RANK = 64
LINEAR_ALPHA = 128


class LinearWorkload:
    """NF4Linear forward + backward with LoRA r=64 at the config-5 micro-benchmark shapes.

    One step, per weight: xa = s x A^T (cuBLAS), y = fused NF4 GEMM(x, W) + xa B^T,
    dyb = s dy B (cuBLAS), dx = fused NF4 dX(dy, W) + dyb A, dA = dyb^T x, dB = dy^T xa
    (cuBLAS) -- exactly the launches NF4Linear's autograd makes.
    """

    def __init__(self, device, T=LINEAR_T):
        from stratum_b200 import functional as F
        from stratum_b200 import ops

        self.F, self.ops, self.device, self.T = F, ops, device, T
        self.scaling = LINEAR_ALPHA / LINEAR_RANK
        g = torch.Generator(device=device).manual_seed(0)
        self.items = []
        for N, K in LINEAR_SHAPES:
            w = (torch.randn(N, K, generator=g, device=device) * 0.02).to(torch.float16)
            packed, qs = F.quantize_4bit(w)
            x = torch.randn(T, K, generator=g, device=device).to(torch.bfloat16)
            dy = torch.randn(T, N, generator=g, device=device).to(torch.bfloat16)
            A = ((torch.rand(LINEAR_RANK, K, generator=g, device=device) * 2 - 1) / K**0.5).to(torch.bfloat16)
            B = (torch.randn(N, LINEAR_RANK, generator=g, device=device) * 0.01).to(torch.bfloat16)
            self.items.append(dict(N=N, K=K, packed=packed, qs=qs, x=x, dy=dy, A=A, B=B,
                                   wbuf=torch.empty(N, K, dtype=torch.bfloat16, device=device)))
        r = LINEAR_RANK
        self.flops_main = sum(4.0 * T * it["N"] * it["K"] for it in self.items)  # fwd + dX
        self.flops_lora = sum(2.0 * T * r * (it["K"] + it["N"]) * 3 for it in self.items)  # fwd, dX, dA/dB

    def step(self, events=None):
        ops, s = self.ops, self.scaling
        for it in self.items:
            ev = lambda: torch.cuda.Event(enable_timing=True, external=True)  # noqa: E731
            xa = ops.lora_down(it["x"], it["A"], s)
            e0 = ev() if events is not None else None
            if e0: e0.record()
            y = ops.nf4_gemm_fwd(it["x"], it["packed"], it["qs"], lora_A=it["A"], lora_B=it["B"], scaling=s, xa=xa)
            if e0:
                e1 = ev(); e1.record(); events.append(("fwd", it["N"], it["K"], e0, e1))
            dyb = ops.lora_down(it["dy"], it["B"].t(), s)
            e0 = ev() if events is not None else None
            if e0: e0.record()
            dx = ops.nf4_gemm_dx(it["dy"], it["packed"], it["qs"], lora_A=it["A"], lora_B=it["B"], scaling=s, dyb=dyb)
            if e0:
                e1 = ev(); e1.record(); events.append(("dx", it["N"], it["K"], e0, e1))
            dA = dyb[:, :LINEAR_RANK].t() @ it["x"]
            dB = it["dy"].t() @ xa[:, :LINEAR_RANK]
            del y, dx, dA, dB

    def unfused_step(self):
        """Reference GPU path: dequantize to bf16, then cuBLAS forward and dX (the reference's K2 + K3)."""
        for it in self.items:
            self.F.dequantize_4bit(it["packed"], it["qs"], out=it["wbuf"], out_dtype=torch.bfloat16)
            torch.matmul(it["x"], it["wbuf"].t())
            torch.matmul(it["dy"], it["wbuf"])


def run_linear_metrics(args, world, flush, clocks_ctx=True):
    """Time LinearWorkload steps (CUDA-graph replays); returns a dict of results."""
    dev = torch.device("cuda", torch.cuda.current_device())
    wl = LinearWorkload(dev)
    ev = []
    g_f, _, launches = capture(lambda: (ev.clear(), wl.step(ev)))
    g_u, _, _ = capture(wl.unfused_step)
    for _ in range(args.warmup):
        g_f.replay()
        g_u.replay()
    torch.cuda.synchronize()

    def timed(graph, n, collect=None):
        out = []
        for _ in range(n):
            flush.fill_(1)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            e1.synchronize()
            out.append(e0.elapsed_time(e1))
            if collect is not None:
                collect += [(k, n_, k_, a.elapsed_time(b)) for k, n_, k_, a, b in ev]
        return out

    barrier(world)
    torch.cuda.synchronize()
    kern = []
    nsteps = max(3, min(args.steps, 30))
    with ClockSampler(dev.index) as clocks:
        step_ms = timed(g_f, nsteps, kern)
        torch.cuda.synchronize()
        barrier(world)
        base_ms = timed(g_u, max(3, nsteps // 3))
    ms = max_over_ranks(statistics.mean(step_ms), world)
    flops = wl.flops_main + wl.flops_lora
    peaks = load_peaks()
    per = {}
    for kind in ("fwd", "dx"):
        for N, K in LINEAR_SHAPES:
            ts = [t for k, n, kk, t in kern if k == kind and n == N and kk == K]
            per[f"{kind} {N}x{K}"] = round(2.0 * LINEAR_T * N * K / (statistics.mean(ts) * 1e-3) / 1e12, 1)
    kflops = sum(2.0 * LINEAR_T * n * k for _, n, k, _ in kern)
    kms = sum(t for _, _, _, t in kern)
    achieved = kflops / (kms * 1e-3) / 1e12
    base = statistics.mean(base_ms)
    return {
        "metric": "nf4_linear_fwd_bwd_TFLOPs",
        "value": round(flops * world / (ms * 1e-3) / 1e12, 1),
        "unit": "TFLOP/s",
        "ms_per_step": round(ms, 4),
        "workload": f"NF4Linear fwd+bwd (fused fwd, fused dX, LoRA r={LINEAR_RANK} grads), T={LINEAR_T}, "
                    "weights 14336x4096 and 4096x14336, bf16 activations",
        "roofline": {"bound": "tensor", "kernel": "k_nf4_gemm_fwd + k_nf4_gemm_dx", "achieved": round(achieved, 1),
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                     "frac_of": peaks["source"], "frac_nominal_2250": round(achieved / 2250.0, 4),
                     "per_kernel_TFLOPs": per, "traffic": None},
        "gpu_reference_path": {"what": "dequantize_4bit -> bf16, cuBLAS forward + cuBLAS dX (no LoRA)",
                               "TFLOPs": round(wl.flops_main / (base * 1e-3) / 1e12, 1), "ms_per_step": round(base, 4)},
        "gpu_launches_per_step": int(launches),
        "clocks": clocks.summary(),
    }


LINEAR_SWEEP = ((1024, 5632, 2048), (2048, 4096, 14336), (4096, 4096, 14336), (8192, 4096, 14336),
                (8192, 14336, 4096))  # (T, N, K): config 1, then the config-5 down-proj shape over T


def run_linear_sweep(flush):
    """Fused NF4 forward + input gradient against the reference's GPU path (dequantize to
    bf16, cuBLAS forward, cuBLAS dX) over token counts, no LoRA on either side: where the
    fused kernels win and by how much.  CUDA-graph replays, L2 flushed between steps."""
    from stratum_b200 import functional as F
    from stratum_b200 import ops

    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(3)
    rows = []
    for T, N, K in LINEAR_SWEEP:
        w = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.float16)
        packed, qs = F.quantize_4bit(w)
        del w
        x = torch.randn(T, K, generator=g, device=dev).to(torch.bfloat16)
        dy = torch.randn(T, N, generator=g, device=dev).to(torch.bfloat16)
        wbuf = torch.empty(N, K, dtype=torch.bfloat16, device=dev)
        y = torch.empty(T, N, dtype=torch.bfloat16, device=dev)
        dx = torch.empty(T, K, dtype=torch.bfloat16, device=dev)

        def fused():
            ops.nf4_gemm_fwd(x, packed, qs, out=y)
            ops.nf4_gemm_dx(dy, packed, qs, out=dx)

        def unfused():
            F.dequantize_4bit(packed, qs, out=wbuf, out_dtype=torch.bfloat16)
            torch.matmul(x, wbuf.t(), out=y)
            torch.matmul(dy, wbuf, out=dx)

        graphs = [capture(fused)[0], capture(unfused)[0]]
        times = []
        for gr in graphs:
            for _ in range(3):
                gr.replay()
            ts = []
            for _ in range(10):
                flush.fill_(1)
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                gr.replay()
                e1.record()
                e1.synchronize()
                ts.append(e0.elapsed_time(e1))
            times.append(statistics.median(ts))
        flops = 4.0 * T * N * K
        rows.append({"T": T, "N": N, "K": K, "fused_TFLOPs": round(flops / (times[0] * 1e-3) / 1e12, 1),
                     "dequant_cublas_TFLOPs": round(flops / (times[1] * 1e-3) / 1e12, 1),
                     "fused_over_unfused": round(times[1] / times[0], 3)})
        del graphs, x, dy, wbuf, y, dx, packed, qs
        torch.cuda.empty_cache()
    return rows


def run_linear(args, world, rank, local):
    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    r = run_linear_metrics(args, world, flush)
    r["sweep_fused_vs_dequant_cublas"] = run_linear_sweep(flush)
    out = {
        "metric": r["metric"], "value": r["value"], "unit": r["unit"], "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (NF4 weights)",
        "data": "synthetic: W ~N(0,0.02) fp16 -> NF4 bs64, x, dY ~N(0,1) bf16, LoRA r=64 alpha=128",
        "config": {"workload": r["workload"], "parallelism": f"replicas x{world}",
                   "l2": "256 MiB fill between timed steps"},
        "roofline": r["roofline"], "gpu_reference_path": r["gpu_reference_path"],
        "sweep_fused_vs_dequant_cublas": r["sweep_fused_vs_dequant_cublas"],
        "gpu_launches": r["gpu_launches_per_step"] * args.steps, "clocks": r["clocks"],
    }
    return out


MOE_T, MOE_E, MOE_TOPK, MOE_H, MOE_I = 4096, 128, 8, 2048, 768  # one Qwen3-30B-A3B-shaped expert layer


class ExpertsWorkload:
    """Routed experts of one Qwen3-30B-A3B-shaped MoE layer, forward + backward.

    4096 tokens, 128 experts, top-8 from a N(0, 0.02) router (data-dependent,
    skewed routing), hidden 2048, expert intermediate 768; expert weights NF4
    bs64.  ``step`` is what NF4Experts' autograd launches (route, gather, grouped
    gate_up + SwiGLU, grouped down, combine; combine grad, grouped dX down, SwiGLU
    grad, grouped dX gate_up, combine), with events around the grouped GEMMs.
    ``module_step`` calls the module itself.  ``reference_step`` is the
    reference's GPU path: dequantize every expert to bf16, then HF
    Qwen3MoeExperts' per-expert loop forward + autograd backward.
    """

    def __init__(self, device):
        from stratum_b200 import functional as F
        from stratum_b200 import ops
        from stratum_b200.experts import NF4Experts

        self.F, self.ops, self.device = F, ops, device
        g = torch.Generator(device=device).manual_seed(0)
        E, H, I, T, k = MOE_E, MOE_H, MOE_I, MOE_T, MOE_TOPK
        holder = torch.nn.Module()
        holder.gate_up_proj = torch.nn.Parameter((torch.randn(E, 2 * I, H, generator=g, device=device) * 0.02).half(),
                                                 requires_grad=False)
        holder.down_proj = torch.nn.Parameter((torch.randn(E, H, I, generator=g, device=device) * 0.02).half(),
                                              requires_grad=False)
        holder.act_fn = torch.nn.SiLU()
        self.mod = NF4Experts.from_experts(holder)
        del holder
        x = torch.randn(T, H, generator=g, device=device).to(torch.bfloat16)
        wr = torch.randn(E, H, generator=g, device=device) * 0.02
        probs = torch.softmax(x.float() @ wr.t(), dim=-1)
        w, idx = torch.topk(probs, k, dim=-1)
        w = w / w.sum(-1, keepdim=True)  # norm_topk_prob
        self.idx = idx
        self.x = x.requires_grad_()
        self.w = w.requires_grad_()
        self.dout = torch.randn(T, H, generator=g, device=device).to(torch.bfloat16)
        counts = torch.bincount(idx.reshape(-1), minlength=E)
        self.tokens_per_expert = {"mean": round(float(counts.float().mean()), 1), "max": int(counts.max()),
                                  "min": int(counts.min())}
        rows = T * k
        self.flops_fwd = 2.0 * rows * (2 * I * H + H * I)
        self.flops = 2.0 * self.flops_fwd  # forward + input gradient (the experts are frozen)
        self.gu_buf = self.dn_buf = self.hf = None

    def module_step(self):
        self.x.grad = None
        self.w.grad = None
        out = self.mod(self.x, self.idx, self.w)
        out.backward(self.dout)

    def step(self, events=None):
        ops, m = self.ops, self.mod
        ev = lambda: torch.cuda.Event(enable_timing=True, external=True)  # noqa: E731

        def start():
            if events is None:
                return None
            e0 = ev()
            e0.record()
            return e0

        def mark(name, e0):
            if events is not None:
                e1 = ev()
                e1.record()
                events.append((name, e0, e1))

        r = ops.moe_route(self.idx, m.num_experts)
        xs = ops.moe_gather_rows(self.x.detach(), r.token_of)
        e0 = start()
        h, gu = ops.nf4_grouped_fwd(xs, r, m.gate_up, m.gate_up_state, swiglu=True, keep_gate_up=True)
        mark("fwd_gate_up_swiglu", e0)
        e0 = start()
        o = ops.nf4_grouped_fwd(h, r, m.down, m.down_state)
        mark("fwd_down", e0)
        w = self.w.detach().reshape(-1)
        ops.moe_combine(o, r, w)
        dys, dw = ops.moe_combine_grad(self.dout, r, w, o)
        e0 = start()
        dh = ops.nf4_grouped_dx(dys, r, m.down, m.down_state)
        mark("dx_down", e0)
        dgu = ops.swiglu_grad(gu, dh)
        e0 = start()
        dxs = ops.nf4_grouped_dx(dgu, r, m.gate_up, m.gate_up_state)
        mark("dx_gate_up", e0)
        ops.moe_combine(dxs, r, None)

    def grouped_mm_step(self, events=None):
        """A fair GPU baseline: dequantize every expert to bf16 (as the reference stages
        them), then cuBLAS-class grouped GEMMs (``torch._grouped_mm``) over the same
        routing, gather, combine and SwiGLU gradient kernels as ours; forward + input
        gradient.  ``events`` collects (name, e0, e1) around the four grouped GEMMs."""
        import torch.nn.functional as TF

        ops, m, F = self.ops, self.mod, self.F
        E, H, I = MOE_E, MOE_H, MOE_I
        if self.gu_buf is None:
            self.gu_buf = torch.empty(E * 2 * I, H, dtype=torch.bfloat16, device=self.device)
            self.dn_buf = torch.empty(E * H, I, dtype=torch.bfloat16, device=self.device)
        F.dequantize_4bit(m.gate_up, m.gate_up_state, out=self.gu_buf, out_dtype=torch.bfloat16)
        F.dequantize_4bit(m.down, m.down_state, out=self.dn_buf, out_dtype=torch.bfloat16)
        wgu = self.gu_buf.view(E, 2 * I, H)
        wdn = self.dn_buf.view(E, H, I)
        ev = lambda: torch.cuda.Event(enable_timing=True, external=True)  # noqa: E731

        def gmm(name, a, b, offs):
            e0 = None
            if events is not None:
                e0 = ev()
                e0.record()
            out = torch._grouped_mm(a, b, offs=offs)
            if events is not None:
                e1 = ev()
                e1.record()
                events.append((name, e0, e1))
            return out

        r = ops.moe_route(self.idx, E)
        offs = r.offsets[1:]
        xs = ops.moe_gather_rows(self.x.detach(), r.token_of)
        gu = gmm("fwd_gate_up", xs, wgu.transpose(-2, -1), offs)
        g, u = gu[:, :I], gu[:, I:]
        h = (TF.silu(g) * u).contiguous()
        o = gmm("fwd_down", h, wdn.transpose(-2, -1), offs)
        w = self.w.detach().reshape(-1)
        ops.moe_combine(o.contiguous(), r, w)
        dys, _ = ops.moe_combine_grad(self.dout, r, w, o.contiguous())
        dh = gmm("dx_down", dys, wdn, offs)
        dgu = ops.swiglu_grad(gu.contiguous(), dh.contiguous())
        dxs = gmm("dx_gate_up", dgu, wgu, offs)
        ops.moe_combine(dxs.contiguous(), r, None)

    def reference_step(self):
        from transformers import Qwen3MoeConfig
        from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeExperts

        E, H, I = MOE_E, MOE_H, MOE_I
        if self.hf is None:
            cfg = Qwen3MoeConfig(hidden_size=H, moe_intermediate_size=I, num_experts=E, num_experts_per_tok=MOE_TOPK,
                                 hidden_act="silu")
            with torch.device("meta"):
                self.hf = Qwen3MoeExperts(cfg)
            self.gu_buf = torch.empty(E * 2 * I, H, dtype=torch.bfloat16, device=self.device)
            self.dn_buf = torch.empty(E * H, I, dtype=torch.bfloat16, device=self.device)
            self.hf.gate_up_proj = torch.nn.Parameter(self.gu_buf.view(E, 2 * I, H), requires_grad=False)
            self.hf.down_proj = torch.nn.Parameter(self.dn_buf.view(E, H, I), requires_grad=False)
        m = self.mod
        self.F.dequantize_4bit(m.gate_up, m.gate_up_state, out=self.gu_buf, out_dtype=torch.bfloat16)
        self.F.dequantize_4bit(m.down, m.down_state, out=self.dn_buf, out_dtype=torch.bfloat16)
        self.x.grad = None
        self.w.grad = None
        out = self.hf(self.x, self.idx, self.w)
        out.backward(self.dout)


def run_experts_metrics(args, world, flush):
    """Time ExpertsWorkload: the module (CUDA-graph replays), the per-kernel split, and the reference path."""
    dev = torch.device("cuda", torch.cuda.current_device())
    wl = ExpertsWorkload(dev)
    ev = []
    g_m, _, launches = capture(wl.module_step)
    g_k, _, _ = capture(lambda: (ev.clear(), wl.step(ev)))
    for _ in range(args.warmup):
        g_m.replay()
        g_k.replay()
        wl.reference_step()
    torch.cuda.synchronize()

    def timed(run, n, collect=None):
        out = []
        for _ in range(n):
            flush.fill_(1)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            run()
            e1.record()
            e1.synchronize()
            out.append(e0.elapsed_time(e1))
            if collect is not None:
                collect += [(name, a.elapsed_time(b)) for name, a, b in ev]
        return out

    barrier(world)
    torch.cuda.synchronize()
    nsteps = max(3, min(args.steps, 30))
    kern = []
    with ClockSampler(dev.index) as clocks:
        mod_ms = timed(g_m.replay, nsteps)
        timed(g_k.replay, nsteps, kern)
        torch.cuda.synchronize()
        barrier(world)
        ref_ms = timed(wl.reference_step, max(3, nsteps // 3))
    ms = max_over_ranks(statistics.mean(mod_ms), world)
    peaks = load_peaks()
    E, H, I, rows = MOE_E, MOE_H, MOE_I, MOE_T * MOE_TOPK
    kflops = {"fwd_gate_up_swiglu": 2.0 * rows * 2 * I * H, "fwd_down": 2.0 * rows * H * I,
              "dx_down": 2.0 * rows * H * I, "dx_gate_up": 2.0 * rows * 2 * I * H}
    per = {}
    tot_f = tot_ms = 0.0
    for name, f in kflops.items():
        t = statistics.mean([t for n, t in kern if n == name])
        per[name] = {"TFLOPs": round(f / (t * 1e-3) / 1e12, 1), "ms": round(t, 4)}
        tot_f += f
        tot_ms += t
    achieved = tot_f / (tot_ms * 1e-3) / 1e12
    ref = statistics.mean(ref_ms)
    # fair baseline: dequantized experts + torch._grouped_mm, CUDA-graph replays like ours
    gmm = None
    try:
        gev = []
        g_g, _, _ = capture(lambda: (gev.clear(), wl.grouped_mm_step(gev)))
        for _ in range(3):
            g_g.replay()
        gkern = []
        gms = statistics.mean(timed(g_g.replay, nsteps))
        for _ in range(nsteps):
            flush.fill_(1)
            g_g.replay()
            torch.cuda.synchronize()
            gkern += [(name, a.elapsed_time(b)) for name, a, b in gev]
        gflops = {"fwd_gate_up": kflops["fwd_gate_up_swiglu"], "fwd_down": kflops["fwd_down"],
                  "dx_down": kflops["dx_down"], "dx_gate_up": kflops["dx_gate_up"]}
        gper = {}
        gf = gt = 0.0
        for name, f in gflops.items():
            t = statistics.mean([t for n, t in gkern if n == name])
            gper[name] = {"TFLOPs": round(f / (t * 1e-3) / 1e12, 1), "ms": round(t, 4)}
            gf += f
            gt += t
        gmm = {"what": "dequantize every expert to bf16, then torch._grouped_mm (bf16, fp32 accumulate) for the "
                       "four expert GEMMs over the same routing, gather, combine and SwiGLU-gradient kernels",
               "layer_TFLOPs": round(wl.flops / (gms * 1e-3) / 1e12, 1), "ms_per_step": round(gms, 4),
               "gemm_TFLOPs": round(gf / (gt * 1e-3) / 1e12, 1), "per_kernel": gper,
               "ours_over_grouped_mm": round(gms / ms, 3)}
        del g_g
    except Exception as exc:  # an unsupported layout or arch is reported, not fatal
        gmm = {"unavailable": f"{type(exc).__name__}: {str(exc).splitlines()[0][:200]}"}
    return {
        "metric": "nf4_moe_experts_fwd_bwd_TFLOPs",
        "value": round(wl.flops * world / (ms * 1e-3) / 1e12, 1),
        "unit": "TFLOP/s",
        "ms_per_step": round(ms, 4),
        "tokens_per_s": round(MOE_T * world / (ms * 1e-3), 1),
        "workload": f"NF4Experts fwd+bwd, one Qwen3-30B-A3B-shaped layer: T={MOE_T}, E={E}, top-{MOE_TOPK}, "
                    f"H={H}, I={I}, N(0,0.02) router",
        "tokens_per_expert": wl.tokens_per_expert,
        "roofline": {"bound": "tensor", "kernel": "k_grouped_fwd + k_grouped_dx", "achieved": round(achieved, 1),
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                     "frac_of": peaks["source"], "per_kernel": per, "traffic": None},
        "gpu_reference_path": {"what": "dequantize every expert to bf16, HF Qwen3MoeExperts per-expert loop fwd + "
                                       "autograd bwd (the reference's path on a GPU)",
                               "TFLOPs": round(wl.flops / (ref * 1e-3) / 1e12, 1), "ms_per_step": round(ref, 4),
                               "speedup": round(ref / ms, 2)},
        "gpu_grouped_mm_path": gmm,
        "gpu_launches_per_step": int(launches),
        "clocks": clocks.summary(),
    }


def run_experts(args, world, rank, local):
    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    r = run_experts_metrics(args, world, flush)
    return {
        "metric": r["metric"], "value": r["value"], "unit": r["unit"], "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (NF4 weights)",
        "data": "synthetic: expert weights ~N(0,0.02) fp16 -> NF4 bs64, x, dY ~N(0,1) bf16, router ~N(0,0.02)",
        "config": {"workload": r["workload"], "parallelism": f"replicas x{world}",
                   "l2": "256 MiB fill between timed steps"},
        "tokens_per_s": r["tokens_per_s"], "tokens_per_expert": r["tokens_per_expert"],
        "roofline": r["roofline"], "gpu_reference_path": r["gpu_reference_path"],
        "gpu_grouped_mm_path": r["gpu_grouped_mm_path"],
        "gpu_launches": r["gpu_launches_per_step"] * args.steps, "clocks": r["clocks"],
    }


PIPE_SEQ = {"llama3-8b": 8192, "qwen3-0.6b": 2048, "qwen3-30b-a3b": 4096}
# postfix (lm_head fwd + dX + cross entropy) cost per microbatch in decoder-layer units, measured
PIPE_TAIL_COST = {"llama3-8b": 1.5, "qwen3-0.6b": 8.0, "qwen3-30b-a3b": 2.0}


def run_pipeline_metrics(args, world, rank, local, model=None, microbatches=None, steps=None, warmup=None):
    """Layer-parallel training step of a BASELINE decoder config through RankPipeline.

    Each rank builds only its stratum (``assign.strata``); config 5 (llama3-8b)
    streams its NF4 + double-quant weights from pinned host every step.  One
    step = forward + backward of ``microbatches`` sequences (GPipe); tokens/s
    counts every sequence's tokens once.  Also times the sequential schedule
    (one sequence per step, the reference's execution) and an end-to-end step
    whose token ids come from pinned host memory and whose loss is read back.
    """
    import torch.distributed as dist

    from stratum_b200 import _lib
    from stratum_b200 import decoder as D
    from stratum_b200.assign import balanced_strata
    from stratum_b200.pipeline import RankPipeline
    from stratum_b200.stage import DeviceStage

    model = model or args.model
    spec = D.SPECS[model]
    seq = PIPE_SEQ[model]
    M = int(microbatches or args.microbatches or 8 * world)
    steps = max(1, int(steps if steps is not None else args.pipe_steps))
    warmup = max(1, int(warmup if warmup is not None else args.pipe_warmup))
    dev = torch.device("cuda", local)
    first, last = rank == 0, rank == world - 1
    # the last rank also runs the postfix (lm_head + cross entropy): give it fewer layers
    strata = balanced_strata(spec.layers, world, tail_cost=PIPE_TAIL_COST[model])
    mine = strata[rank]
    n_layers_of = [len(x) for x in strata]
    stream = model == "llama3-8b"  # config 5: weights streamed per step from pinned host
    sink = D.RouterLogitsSink() if spec.experts else None
    t_build = time.perf_counter()
    layers = [D.WrappedLayer(D.build_layer(spec, i, dev, stream=stream, seed=0, sink=sink), i) for i in mine]
    prefix = D.Prefix(spec, dev, seed=0, with_embedding=first)
    postfix = D.Postfix(spec, dev, seed=0) if last else None
    t_build = time.perf_counter() - t_build
    # 1F1B keeps at most world - rank microbatches in flight, so every layer's graph is kept (no
    # recompute); the router aux loss's per-microbatch sums ride on the boundary messages
    schedule, recompute = "1f1b", False
    # one GPU with resident weights and no router aux loss: microbatches replay a CUDA graph
    graphed = world == 1 and not stream and not (spec.experts and spec.router_aux_coef)
    pipe = RankPipeline(DeviceStage(layers, local), prefix=prefix, postfix=postfix, rank=rank, world=world,
                        hidden_size=spec.hidden, router_sink=sink, router_aux_coef=spec.router_aux_coef,
                        n_experts=spec.experts, schedule=schedule, recompute=recompute, cuda_graph=graphed)
    g = torch.Generator(device=dev).manual_seed(1234)
    ids = torch.randint(0, spec.vocab, (M, seq), generator=g, device=dev)
    ids_host = ids.cpu().pin_memory()

    def step(mb, host=False):
        src = ids_host if host else ids
        out = pipe.train_step(src[:mb] if first else None, src[:mb] if last else None, microbatches=mb,
                              seq_len=seq)
        return out

    timed_own_ms = []
    # a step whose kernels report that a bounded device-side wait gave up (the status word
    # read at the end of train_step) is run again by train_step (or raises once its retries
    # are spent) and carries a ~2 s stall in its time: the attempt is discarded and timed
    # again (at most twice), and the line says how many were
    status_errors = {"discarded_attempts": 0, "errors_in_reported": 0, "warmup_errors": 0, "last": ""}

    def guarded(mb, host=False):
        try:
            loss = step(mb, host)
            if host and loss is not None:
                float(loss)  # the step's result read back to the host
            return 0
        except _lib.StratumError as exc:
            status_errors["last"] = str(exc)[:300]
            print(f"[bench] rank {rank}: {exc}", file=sys.stderr, flush=True)
            return 1

    def timed(mb, n, host=False):
        for attempt in range(3):
            barrier(world)
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            n0, g0, r0 = _lib.launch_count(), pipe.graph_launches, pipe.status_retries
            e0.record()
            bad = 0
            for _ in range(n):
                bad += guarded(mb, host)
            e1.record()
            torch.cuda.synchronize()
            launches = _lib.launch_count() - n0 + pipe.graph_launches - g0
            bad += pipe.status_retries - r0  # steps train_step itself ran again
            barrier(world)
            bad = int(max_over_ranks(float(bad), world))
            if bad == 0 or attempt == 2:
                break
            status_errors["discarded_attempts"] += 1
        status_errors["errors_in_reported"] += bad
        timed_own_ms.append(e0.elapsed_time(e1) / n)
        return max_over_ranks(e0.elapsed_time(e1) / n, world), launches

    for _ in range(warmup):
        status_errors["warmup_errors"] += guarded(M)
    if graphed:
        step(1)  # the sequential schedule's graph, built outside its timing
    torch.cuda.synchronize()
    # the boundary receives' stream waits are bracketed by CUDA events during the timed steps
    pipe.chan.wait_events = []
    with ClockSampler(dev.index) as clocks:
        ms, launches = timed(M, steps)
    own_ms = timed_own_ms[-1]
    wait_ms = sum(a.elapsed_time(b) for a, b in pipe.chan.wait_events) / steps
    pipe.chan.wait_events = None
    per_rank = torch.tensor([own_ms, wait_ms], dtype=torch.float64, device=dev)
    if world > 1:
        gathered = [torch.empty_like(per_rank) for _ in range(world)]
        dist.all_gather(gathered, per_rank)
    else:
        gathered = [per_rank]
    ranks = [{"rank": r, "layers": n_layers_of[r], "step_ms": round(float(t[0]), 2),
              "boundary_wait_ms": round(float(t[1]), 2), "busy_ms": round(float(t[0] - t[1]), 2)}
             for r, t in enumerate(gathered)]
    ms_seq, _ = timed(1, max(1, steps))
    ms_e2e, _ = timed(M, 1, host=True)
    tok = M * seq
    value = tok / (ms * 1e-3)
    peaks = load_peaks()
    fpt = D.reference_flops_per_token(spec, seq)
    achieved = fpt * value / 1e12
    peak = peaks.get("bf16_tflops_sustained") or peaks["bf16_tflops"]
    lt = torch.tensor([launches], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(lt)
    # what bounds the step: the 1F1B schedule leaves each rank idle for N - 1 of M + N - 1
    # microbatch slots; boundary waits above that share are imbalance or transfer time
    bubble = (world - 1) / (M + world - 1)  # idle share of a rank under 1F1B (and GPipe) with M microbatches
    worst_wait = max(r["boundary_wait_ms"] / max(r["step_ms"], 1e-9) for r in ranks)
    busiest = max(ranks, key=lambda r: r["busy_ms"])
    if world == 1:
        limiter = "compute (one rank, no boundaries)"
    elif worst_wait <= bubble + 0.05:
        limiter = (f"1F1B bubble: boundary waits <= {worst_wait:.1%} of the step against a predicted "
                   f"{bubble:.1%}; the busiest rank ({busiest['rank']}) computes {busiest['busy_ms']} ms")
    else:
        limiter = (f"stage imbalance or transfers: a rank waits {worst_wait:.1%} of the step on boundaries, "
                   f"above the {bubble:.1%} bubble; busiest rank {busiest['rank']} computes {busiest['busy_ms']} ms")
    del pipe, layers, prefix, postfix
    torch.cuda.empty_cache()
    return {
        "metric": "pipeline_train_tokens_per_s",
        "value": round(value, 1),
        "unit": "tokens/s",
        "ms_per_step": round(ms, 3),
        "model": model,
        "workload": f"{model}-shaped decoder fwd+bwd, {spec.layers} layers over {world} GPU(s) (one stratum per "
                    f"rank, last rank lighter by the postfix), {M} microbatches x [1, {seq}] tokens per step ({schedule}, "
                    f"{'per-layer recompute' if recompute else 'no recompute'}), NF4 bs64"
                    f"{' + double quant, streamed per step from pinned host' if stream else ' resident'}, "
                    f"LoRA r={spec.lora_r}, NCCL send/recv boundaries"
                    f"{'; microbatches replayed from a CUDA graph of one forward + backward' if graphed else ''}",
        "microbatches": M,
        "seq_len": seq,
        "sequential": {"what": "one sequence per step (the reference's sequential execution)",
                       "value": round(seq / (ms_seq * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(ms_seq, 3)},
        "e2e": {"value": round(tok / (ms_e2e * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(ids_host[:M].numel() * 8 * 2),  # token ids and labels
                "d2h_bytes_per_step": 4, "path": "RankPipeline.train_step with pinned host token ids, loss read back"},
        "roofline": {"bound": "tensor", "what": "algorithmic FLOPs of the step (fwd + dX + LoRA grads + attention "
                     "+ lm_head; recompute not counted) per second over all GPUs",
                     "achieved": round(achieved, 1), "peak": round(peak * world, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / (peak * world), 4),
                     "frac_of": f"{peaks['source']} sustained bf16 x {world}", "flops_per_token": fpt},
        "gpu_launches_per_step": int(lt.item() / steps),
        "steps": steps,
        "warmup": warmup,
        "per_rank": ranks,
        "bubble_predicted": round(bubble, 4),
        "limiter": limiter,
        "build_s": round(t_build, 1),
        "clocks": clocks.summary(),
        "device_status": status_errors,
    }


def run_pipeline(args, world, rank, local):
    r = run_pipeline_metrics(args, world, rank, local)
    if rank != 0:
        return None
    return {
        "metric": r["metric"], "value": r["value"], "unit": r["unit"], "n_gpus": world, "steps": args.pipe_steps,
        "warmup": args.pipe_warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (NF4 weights)",
        "data": "synthetic: random-init weights of the named shape, uniform token ids",
        "config": {"workload": r["workload"], "model": r["model"], "global_batch": r["microbatches"],
                   "seq_len": r["seq_len"], "parallelism": f"pp{world}",
                   "l2": "inputs far larger than L2 (the step streams every layer's weights and activations)"},
        "sequential": r["sequential"], "e2e": r["e2e"], "roofline": r["roofline"],
        "gpu_launches": r["gpu_launches_per_step"] * args.pipe_steps, "build_s": r["build_s"], "clocks": r["clocks"],
    }


def run_codec_e2e(args, wl, world):
    """Same work as ``value``, end to end through the reference-facing call with host buffers.

    Each step takes the eight NF4 payloads of the codec workload (the four
    matrices with a plain absmax, then with a double-quantized absmax) from pinned
    host memory: payload i is copied host -> device on a copy stream (one
    ``cudaMemcpyAsync`` per tensor), then ``functional.dequantize_4bit`` turns it
    into bf16 on the compute stream after an event, so payload i+1's copy overlaps
    payload i's dequant; a 4 KiB slice of each result is read back to pinned host.
    The step is timed on the host around a device synchronisation.  The pinned
    H2D rate of the same bytes in one copy is measured beside it: the copies, not
    the dequant, bound this number.
    """
    F = wl.F
    from stratum_b200.functional import QuantState

    dev = wl.device
    payloads = []  # (host tensors, device tensors, build state, out)
    for kind in ("plain", "dq"):
        for it in wl.items:
            if kind == "plain":
                st = it["st"]
                host = [it["packed"], st.absmax]
            else:
                st = it["st_dq"]
                host = [it["packed_dq"], st.absmax, st.state2.absmax, st.offset.reshape(1), st.state2.code]
            host = [h.cpu().pin_memory() for h in host]
            devt = [torch.empty_like(h, device=dev) for h in host]
            if kind == "plain":
                qs = QuantState(devt[1], st.shape, st.code, 64, "nf4", st.dtype)
            else:
                s2 = QuantState(devt[2], code=devt[4], blocksize=st.state2.blocksize, dtype=torch.float32)
                qs = QuantState(devt[1], st.shape, st.code, 64, "nf4", st.dtype, offset=devt[3].reshape(()),
                                state2=s2)
            out = torch.empty(st.shape, dtype=torch.bfloat16, device=dev)
            payloads.append((host, devt, qs, out))
    readback = torch.empty(len(payloads) * 2048, dtype=torch.bfloat16).pin_memory()
    h2d = sum(h.numel() * h.element_size() for hs, _, _, _ in payloads for h in hs)
    d2h = readback.numel() * 2
    copy_stream = torch.cuda.Stream(dev)
    comp = torch.cuda.current_stream(dev)

    def step():
        copy_stream.wait_stream(comp)  # the previous step's dequants are done with the device buffers
        evs = []
        with torch.cuda.stream(copy_stream):
            for hs, ds, _, _ in payloads:
                for h, d in zip(hs, ds):
                    d.copy_(h, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_stream)
                evs.append(ev)
        for i, ((_, ds, qs, out), ev) in enumerate(zip(payloads, evs)):
            comp.wait_event(ev)
            F.dequantize_4bit(ds[0], qs, out=out, out_dtype=torch.bfloat16)
            readback[i * 2048:(i + 1) * 2048].copy_(out.view(-1)[-2048:], non_blocking=True)
        comp.synchronize()

    for _ in range(max(1, args.warmup)):
        step()
    barrier(world)
    n = max(3, min(args.steps, 20))
    t = time.perf_counter()
    for _ in range(n):
        step()
    dt = (time.perf_counter() - t) / n
    dt = max_over_ranks(dt, world)
    # pinned H2D of the same bytes as one copy (the bound of this path)
    big_h = torch.empty(h2d, dtype=torch.uint8).pin_memory()
    big_d = torch.empty(h2d, dtype=torch.uint8, device=dev)
    big_d.copy_(big_h, non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        big_d.copy_(big_h, non_blocking=True)
    e1.record()
    e1.synchronize()
    h2d_rate = h2d * 5 / (e0.elapsed_time(e1) * 1e-3) / 1e9
    del big_h, big_d
    return {"value": round(wl.dequant_bytes * world / dt / 1e9, 2), "unit": "GB/s", "ms_per_step": round(dt * 1e3, 3),
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "h2d_GBps": round(h2d / dt / 1e9, 2), "pinned_h2d_GBps": round(h2d_rate, 2),
            "h2d_frac_of_pinned": round(h2d / dt / 1e9 / h2d_rate, 3),
            "path": "functional.dequantize_4bit of the eight codec payloads (plain and double-quant absmax) from "
                    "pinned host, per-tensor H2D copies on a copy stream overlapped with the dequants"}


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
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("codec", "linear", "experts", "pipeline"), default="codec")
    ap.add_argument("--model", choices=("llama3-8b", "qwen3-0.6b", "qwen3-30b-a3b"), default="llama3-8b",
                    help="decoder config of the pipeline workload / section")
    ap.add_argument("--microbatches", type=int, default=0, help="pipeline microbatches per step (default 8 x GPUs)")
    ap.add_argument("--pipe-steps", type=int, default=5)
    ap.add_argument("--pipe-warmup", type=int, default=3)
    ap.add_argument("--no-pipeline", action="store_true", help="skip the pipeline sections of the codec run")
    ap.add_argument("--no-pipeline-configs", action="store_true",
                    help="skip the config-3 (Qwen3-0.6B) and config-4 (Qwen3-30B-A3B MoE) pipeline sections")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-linear", action="store_true", help="skip the NF4Linear fwd+bwd section of the codec run")
    ap.add_argument("--no-experts", action="store_true", help="skip the MoE experts section of the codec run")
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
            run = {"codec": run_codec, "linear": run_linear, "experts": run_experts,
                   "pipeline": run_pipeline}[args.workload]
            out = run(args, world, rank, local)
        if rank == 0 and out is not None:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
