#!/usr/bin/env python
"""Benchmark driver: FP16 GEMM TFLOP/s on B200, one JSON line.

Default workload (N=1): configuration 2 of the reference's baseline, the
4096^3 fp16 GEMM with fused BiasGeLU (tanh) epilogue and fp16 output, on
synthetic seeded inputs resident in HBM.  A step is one launch of the GEMM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config 1..5]
                  [--impl pax|reference] [--gather]

With N > 1 (launched under torchrun, one rank per GPU) the GEMM is split
along N: rank p owns the column slab [p*Ns, (p+1)*Ns) of B, bias and C with
Ns = N of the configuration (weak scaling: per-GPU work is fixed), and
--gather adds an NCCL all-gather of the C slabs into a replicated C.
`value` = total FLOPs of all ranks / max-over-ranks device time.

--impl reference times the reference's own CPU GEMM (cpu_gemm_ref of
src/host_bridge.c, compiled from its sources into oracle/_ref) on all host
cores over a bounded row sample of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "FP16 GEMM TFLOP/s & % of B200 dense peak (4096³ BiasGeLU); 1/2/4/8-GPU scaling"
CONFIGS = {
    1: dict(M=1024, N=1024, K=1024, epi="none", dist="uniform", name="C1: 1024^3 fp16 GEMM, no epilogue"),
    2: dict(M=4096, N=4096, K=4096, epi="bias_gelu_tanh", dist="uniform",
            name="C2: 4096^3 fp16 GEMM + BiasGeLU(tanh), fp16 out"),
    3: dict(M=16384, N=16384, K=4096, epi="residual_gelu_erf", dist="normal",
            name="C3: M16384 K4096 N16384 + ResidualGeLU(erf), fp16 out"),
    4: dict(M=16, N=16384, K=4096, epi="bias", dist="normal", name="C4: M16 K4096 N16384 + Bias, fp16 out"),
    5: dict(M=32768, N=32768, K=32768, epi="bias_gelu_tanh", dist="uniform",
            name="C5: 32768^3 fp16 GEMM + BiasGeLU(tanh), fp16 out"),
}
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="pax", choices=["pax", "reference"])
    ap.add_argument("--gather", action="store_true")
    ap.add_argument("--gather-impl", default="fused", choices=["fused", "nccl"],
                    help="fused: the GEMM epilogue stores each tile to every peer over NVLink; nccl: all-gather after")
    ap.add_argument("--strong", action="store_true",
                    help="split the configuration's N over the ranks (fixed total work) instead of N per rank")
    ap.add_argument("--seed", type=int, default=0x5EED)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--epilogue", default=None, help="override the configuration's epilogue (diagnostics)")
    ap.add_argument("--m", type=int, default=None, help="override the configuration's M (diagnostics)")
    ap.add_argument("--no-subrecords", action="store_true",
                    help="headline only: skip the other configurations, the collective and the sustained run")
    return ap.parse_args()


def config_for(args) -> dict:
    """The selected configuration with the diagnostic overrides applied; a
    line measured with an override names it in its workload."""
    cfg = dict(CONFIGS[args.config])
    if args.epilogue:
        cfg["epi"] = args.epilogue
        cfg["name"] += f" [epilogue overridden: {args.epilogue}]"
    if args.m is not None:
        if args.m < 1:
            raise SystemExit("--m must be positive")
        cfg["M"] = args.m
        cfg["name"] += f" [M overridden: {args.m}]"
    return cfg


def rank_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(
        os.environ.get("LOCAL_RANK", "0"))


# ------------------------------------------------------------------ CPU legs
def cpu_reference_lib():
    """(callable(A,B,C,m,n,k), kind): the reference build if present, else the port."""
    import oracle

    L = oracle.ref_lib()
    if L is not None:
        return L.paxref_cpu_gemm_ref, "reference"
    O = oracle.lib()
    return O.oracle_cpu_gemm_ref, "port"


def cpu_gemm_sample(cfg, seconds: float, seed: int, threads: int | None = None):
    """Time cpu_gemm_ref on a row sample of the workload using all host cores.

    Rows are split into blocks, one ctypes call per block (the GIL is released
    during the call).  Returns (TFLOP/s, seconds, rows, threads, kind, flops).
    """
    import numpy as np

    fn, kind = cpu_reference_lib()
    M, N, K = cfg["M"], cfg["N"], cfg["K"]
    rng = np.random.default_rng(seed)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float16).astype(np.float32)
    threads = threads or os.cpu_count() or 1
    # calibrate on one row
    a1 = rng.uniform(-1, 1, (1, K)).astype(np.float16).astype(np.float32)
    c1 = np.empty((1, N), np.float32)
    t0 = time.perf_counter()
    fn(a1.ctypes.data, B.ctypes.data, c1.ctypes.data, 1, N, K)
    t_row = max(time.perf_counter() - t0, 1e-6)
    rows = int(max(threads, min(M, seconds * threads / t_row)))
    rows = max(threads, (rows // threads) * threads)
    rows = min(rows, M) if M >= threads else M
    A = rng.uniform(-1, 1, (rows, K)).astype(np.float16).astype(np.float32)
    C = np.empty((rows, N), np.float32)
    per = (rows + threads - 1) // threads
    blocks = [(r0, min(per, rows - r0)) for r0 in range(0, rows, per)]

    def work(b):
        r0, nr = b
        fn(A[r0:].ctypes.data, B.ctypes.data, C[r0:].ctypes.data, nr, N, K)

    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=len(blocks)) as ex:
        list(ex.map(work, blocks))
    dt = time.perf_counter() - t0
    flops = 2.0 * rows * N * K
    return flops / dt / 1e12, dt, rows, len(blocks), kind, flops


def run_reference(args):
    rank, world, _ = rank_env()
    if rank != 0:
        return 0
    cfg = config_for(args)
    per_step = max(2.0, min(args.cpu_seconds, 150.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        cpu_gemm_sample(cfg, per_step, args.seed)
    vals, secs = [], []
    rows = threads = 0
    kind = ""
    for i in range(args.steps):
        v, dt, rows, threads, kind, _ = cpu_gemm_sample(cfg, per_step, args.seed + i)
        vals.append(v)
        secs.append(dt)
    value = statistics.mean(vals)
    sample = (f"{rows} of {cfg['M']} rows of {cfg['name']} per step (cpu_gemm_ref i-j-l fp32 loop, fp32 inputs "
              f"widened from fp16), {threads} row blocks in parallel")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * statistics.mean(secs),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded uniform[-1,1] fp16 widened to fp32)",
        "config": workload_config(cfg, world, args),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(cfg, world, args):
    n_total = cfg["N"] if getattr(args, "strong", False) else cfg["N"] * world
    return {
        "workload": cfg["name"],
        "M": cfg["M"],
        "N_per_gpu": n_total // world,
        "N_total": n_total,
        "K": cfg["K"],
        "epilogue": cfg["epi"],
        "inputs": cfg["dist"],
        "parallelism": f"N-split over {world} GPU(s)" + (
            "" if not args.gather else " + all-gather of C fused into the GEMM epilogue (TMA stores to peers over NVLink)"
            if args.gather_impl == "fused" else " + NCCL all-gather of C"),
        "l2": "flushed between steps (256 MiB write, then 256 MiB read of another buffer)",
        "timing": "CUDA events around each launch; all steps queued behind a device sleep (no host gaps)",
    }


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling during the timed region (the recipe's clocks line)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.idx)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, pw, reasons = [], 0.0, [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
                pw.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        loaded = [s for s, p in zip(sm, pw) if p >= 0.5 * max(pw)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(pw)}


class NvmlSampler:
    """SM clock, power and clock-event reasons of one GPU through NVML (the
    library nvidia-smi reads), polled on a thread with `interval` seconds
    between samples (a sample itself takes about 0.1 ms).  Each sample
    carries its host time, so `stop(window)` can keep only the samples taken
    while the timed steps ran on the GPU.  A timed region of a few
    milliseconds is invisible to a 50 ms nvidia-smi loop; at 0.1 ms between
    samples a 20-step headline region (about 5 ms with its L2 flushes) gets
    20 or more.  The timed steps are queued on the device before the region
    starts, so the polling thread cannot delay them."""

    REASONS = {  # reported name -> NVML bit (clocks_event_reasons.*)
        "hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
        "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
        "hw_power_brake_slowdown": "nvmlClocksEventReasonHwPowerBrakeSlowdown",
        "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
        "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
        "applications_clocks_setting": "nvmlClocksEventReasonApplicationsClocksSetting",
        "gpu_idle": "nvmlClocksEventReasonGpuIdle",
    }

    def __init__(self, pci_bus_id: str | None = None, index: int = 0, interval: float = 0.0001, nvml=None):
        if nvml is None:
            import pynvml as nvml
        self.nv = nvml
        self.nv.nvmlInit()
        self.h = (self.nv.nvmlDeviceGetHandleByPciBusId(pci_bus_id) if pci_bus_id
                  else self.nv.nvmlDeviceGetHandleByIndex(index))
        self.max_mhz = float(self.nv.nvmlDeviceGetMaxClockInfo(self.h, self.nv.NVML_CLOCK_SM))
        self.bits = {name: getattr(self.nv, attr) for name, attr in self.REASONS.items() if hasattr(self.nv, attr)}
        self.interval = interval
        self.samples: list[tuple[float, float, float, int]] = []  # (host time, SM MHz, W, reason mask)
        self._stop = threading.Event()
        self._t = None

    def _poll(self):
        nv, h = self.nv, self.h
        while not self._stop.is_set():
            t = time.perf_counter()
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                mask = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
            except Exception:  # a failed query loses one sample, not the run
                time.sleep(self.interval)
                continue
            self.samples.append((t, sm, pw, mask))
            time.sleep(self.interval)

    def start(self):
        self._t = threading.Thread(target=self._poll, daemon=True)
        self._t.start()

    def stop(self, window: tuple[float, float] | None = None):
        """Summary of the samples whose host time lies in `window` (all of
        them when None).  If none does, the sample nearest the window's
        middle stands in, and `samples_in_window` says 0."""
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=5)
        try:
            self.nv.nvmlShutdown()
        except Exception:
            pass
        if not self.samples:
            return None
        sel = self.samples
        if window is not None:
            sel = [s for s in self.samples if window[0] <= s[0] <= window[1]]
            if not sel:
                mid = 0.5 * (window[0] + window[1])
                sel = [min(self.samples, key=lambda s: abs(s[0] - mid))]
        mask = 0
        for s in sel:
            mask |= s[3]
        in_window = len([s for s in self.samples if window is None or window[0] <= s[0] <= window[1]])
        return {"sm_mhz": statistics.median(s[1] for s in sel), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(n for n, b in self.bits.items() if mask & b and n != "gpu_idle"),
                "samples": len(sel), "samples_in_window": in_window, "power_w_max": max(s[2] for s in sel),
                "source": f"NVML, {self.interval * 1e3:g} ms between samples, samples inside the timed region"}


def clock_sampler(dev_index: int):
    """NVML sampler for the CUDA device `dev_index` (matched by PCI bus id),
    else the nvidia-smi loop."""
    try:
        import torch

        p = torch.cuda.get_device_properties(dev_index)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        return NvmlSampler(pci_bus_id=bus)
    except Exception:
        return ClockSampler(dev_index)


# ------------------------------------------------------------------ GPU leg
def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0, "fallback"


def traffic_from_profiles(config: int):
    """DRAM bytes per launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", f"traffic_c{config}.txt")
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


def decode_stream(A, bias, cfg, K, N, alg_bytes, hbm, flush, dev, layers: int = 8, reps: int = 20):
    """The decode case the skinny kernel is for: `layers` M=16 GEMMs back to
    back, each with its own weights (together 8 x 134 MB, far above L2, so
    every launch streams its B from HBM).  Consecutive launches overlap
    through programmatic dependent launch: a launch's prologue and its first
    ring of B (weights, marked PAX_GEMM_B_CONST) load during the previous
    launch's tail.  Timed per chain with
    CUDA events (L2 flushed before each chain); reported per GEMM."""
    import torch

    import pax_b200

    g = torch.Generator(device=dev)
    g.manual_seed(0xDEC0)
    Bs = [(torch.randn((K, N), generator=g, device=dev) * 0.02).half() for _ in range(layers)]
    Cs = [torch.empty((A.shape[0], N), dtype=torch.float16, device=dev) for _ in range(layers)]
    # Decode weights are never written by the previous GEMM: PAX_GEMM_B_CONST
    # lets each launch start streaming its B before the previous one ends.
    kw = dict(epilogue=cfg["epi"], bias=bias if "bias" in cfg["epi"] else None, b_const=True)

    def chain():
        for B, C in zip(Bs, Cs):
            pax_b200.gemm(A, B, out=C, **kw)

    for _ in range(3):
        flush.zero_()
        chain()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    torch.cuda._sleep(int(0.02 * 2.0e9))
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        chain()
        e1.record()
    torch.cuda.synchronize()
    per = statistics.mean(e0.elapsed_time(e1) for e0, e1 in ev) / layers
    gbs = alg_bytes / (per * 1e-3) / 1e9
    del Bs, Cs
    return {"launches_per_chain": layers, "us_per_gemm": per * 1e3, "achieved": gbs, "frac": gbs / hbm,
            "pdl": os.environ.get("PAX_PDL", "1") != "0", "b_const": True}


def decode_batched(A, bias, cfg, K, N, alg_bytes, hbm, flush, dev, items: int = 8, reps: int = 20):
    """The same decode shape as `items` independent problems (one activation
    and weight matrix each, as for the experts or heads of one layer) in one
    pax_gemm_batched_ex launch: the skinny kernel streams all items' weights
    back to back.  Timed per launch with CUDA events (L2 flushed before
    each); reported per item."""
    import torch

    import pax_b200

    g = torch.Generator(device=dev)
    g.manual_seed(0xBA7C)
    M = A.shape[0]
    As = torch.randn((items, M, K), generator=g, device=dev).half()
    Bs = (torch.randn((items, K, N), generator=g, device=dev) * 0.02).half()
    biases = bias.unsqueeze(0).repeat(items, 1)
    Cs = torch.empty((items, M, N), dtype=torch.float16, device=dev)
    kw = dict(epilogue=cfg["epi"], bias=biases if "bias" in cfg["epi"] else None, out=Cs)
    for _ in range(3):
        flush.zero_()
        pax_b200.gemm_batched(As, Bs, **kw)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    torch.cuda._sleep(int(0.02 * 2.0e9))
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        pax_b200.gemm_batched(As, Bs, **kw)
        e1.record()
    torch.cuda.synchronize()
    per = statistics.mean(e0.elapsed_time(e1) for e0, e1 in ev) / items
    gbs = alg_bytes / (per * 1e-3) / 1e9
    del As, Bs, Cs
    return {"items_per_launch": items, "us_per_gemm": per * 1e3, "achieved": gbs, "frac": gbs / hbm}


def make_operands(cfg, M, N, K, dev, seed, rank=0):
    """Seeded synthetic operands of a configuration on the device: A is the
    same on every rank; B, bias and residual are this rank's column slab."""
    import torch

    ga = torch.Generator(device=dev)
    ga.manual_seed(seed)  # A is replicated: same on every rank
    g = torch.Generator(device=dev)
    g.manual_seed(seed + 1000 * (rank + 1))  # this rank's column slab of B, bias
    if cfg["dist"] == "uniform":
        A = (torch.rand((M, K), generator=ga, device=dev) * 2 - 1).half()
        B = (torch.rand((K, N), generator=g, device=dev) * 2 - 1).half()
    else:
        A = torch.randn((M, K), generator=ga, device=dev).half()
        B = (torch.randn((K, N), generator=g, device=dev) * 0.02).half()
    bias = torch.randn((N,), generator=g, device=dev).half()
    res = torch.randn((M, N), generator=g, device=dev).half() if "residual" in cfg["epi"] else None
    return A, B, bias, res


class L2Flush:
    """Between steps: write a buffer larger than L2, then read a second one,
    so the dirty lines are written back before the timed launch rather than
    during it."""

    def __init__(self, dev):
        import torch

        self.w = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.r = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def zero_(self):
        self.w.zero_()
        self.r.sum()


def timed_steps(step, steps, warmup, flush, dev, world, local):
    """`warmup` untimed steps, then exactly `steps` timed ones, each preceded
    by an L2 flush and bracketed by CUDA events on the current stream.  The
    timed loop is queued behind a device-side sleep, so no host launch
    latency falls between a start and a stop event; a barrier and a
    synchronize come before and after it.  Returns the per-step times, the
    max over ranks of their mean, and the clock samples taken inside the
    timed region."""
    import torch
    import torch.distributed as dist

    for _ in range(warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    # Host cost of enqueueing one step, to size the device-side sleep.
    t0 = time.perf_counter()
    for _ in range(2):
        flush.zero_()
        step()
    host_step = (time.perf_counter() - t0) / 2
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    gate_s = min(2.0, 2.0 * host_step * steps + 0.01)
    clocks = clock_sampler(local)
    clocks.start()
    time.sleep(0.3)
    # The device is idle here, so `anchor` completes as soon as it is
    # recorded: its host time maps event times to host times, which picks
    # out the clock samples taken while the timed steps ran.
    anchor = torch.cuda.Event(enable_timing=True)
    anchor.record()
    t_anchor = time.perf_counter()
    torch.cuda.nvtx.range_push("timed steps")
    torch.cuda._sleep(int(gate_s * 2.0e9))  # ~cycles at up to 2 GHz
    for i in range(steps):
        flush.zero_()
        starts[i].record()
        step()
        stops[i].record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    window = (t_anchor + anchor.elapsed_time(starts[0]) * 1e-3, t_anchor + anchor.elapsed_time(stops[-1]) * 1e-3)
    clk = clocks.stop(window) if isinstance(clocks, NvmlSampler) else clocks.stop()
    ms = [a.elapsed_time(b) for a, b in zip(starts, stops)]
    mean = statistics.mean(ms)
    t = torch.tensor([mean], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if clk is not None:
        # Cycles per step at the median SM clock of the timed region.
        clk["kcycles_per_step_at_median"] = mean * clk["sm_mhz"]
        clk["step_ms"] = {"first": [round(x, 5) for x in ms[:5]], "last": [round(x, 5) for x in ms[-5:]],
                          "median": statistics.median(ms), "min": min(ms), "max": max(ms)}
    return {"ms": ms, "mean": mean, "max_over_ranks": float(t.item()), "clocks": clk}


def kernel_name(A, B, C, **kw):
    """Which kernel pax_gemm_ex runs for the problem (host-side queries)."""
    import pax_b200

    algo = pax_b200.select_algo(A, B, C, **kw).name.lower()
    d = pax_b200.make_desc(A, B, C, **kw)
    smem = int(pax_b200.lib.pax_gemm_smem_bytes(ctypes.byref(d)))
    return {"algo": algo, "stages": pax_b200.pipeline_stages(A, B, C, **kw), "dynamic_smem_bytes": smem}


def lean_bound(frac, stages):
    return {"stages": stages, "bound_frac": (1 - 1 / stages) if stages else None, "measured_frac_of_roof": frac,
            "holds": (frac >= 1 - 1 / stages) if (frac is not None and stages) else None}


def config_record(cfg_id, args, dev, flush, peak, hbm, steps, warmup):
    """Device-timed sub-record of one configuration at N=1: ms per launch,
    TFLOP/s, roofline fraction against the measured peaks, the committed
    ncu DRAM traffic over the algorithmic bytes, the Lean pipeline-bound
    check and the clocks of its timed region."""
    import torch

    import pax_b200

    cfg = CONFIGS[cfg_id]
    M, N, K = cfg["M"], cfg["N"], cfg["K"]
    A, B, bias, res = make_operands(cfg, M, N, K, dev, args.seed)
    C = torch.empty((M, N), dtype=torch.float16, device=dev)
    kw = dict(epilogue=cfg["epi"], bias=bias if "bias" in cfg["epi"] else None, residual=res)
    r = timed_steps(lambda: pax_b200.gemm(A, B, out=C, **kw), steps, warmup, flush, dev, 1, dev.index)
    flops = 2.0 * M * N * K
    alg_bytes = 2 * (M * K + K * N + M * N) + (2 * N if "bias" in cfg["epi"] else 0) + (
        2 * M * N if res is not None else 0)
    tf = flops / (r["mean"] * 1e-3) / 1e12
    traffic = traffic_from_profiles(cfg_id)
    info = kernel_name(A, B, C, **kw)
    rec = {"workload": cfg["name"], "steps": steps, "warmup": warmup, "ms_per_launch": r["mean"],
           "best_ms": min(r["ms"]), "tflops": tf, "kernel": info, "clocks": r["clocks"]}
    if cfg_id == 4:
        gbs = alg_bytes / (r["mean"] * 1e-3) / 1e9
        rec["roofline"] = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                           "algorithmic_bytes_per_launch": alg_bytes, "traffic": traffic,
                           "traffic_over_algorithmic": traffic / alg_bytes if traffic else None}
        rec["single"] = {"us_per_gemm": r["mean"] * 1e3, "achieved": gbs, "frac": gbs / hbm}
        # The same event pair around an empty launch (torch's one-thread
        # spin kernel, 1 cycle), after the same L2 flush: the fixed cost an
        # isolated, event-timed launch carries whatever the kernel does.
        fl = timed_steps(lambda: torch.cuda._sleep(1), steps, warmup, flush, dev, 1, dev.index)
        above = r["mean"] - fl["mean"]
        rec["single"]["empty_launch_us"] = fl["mean"] * 1e3
        rec["single"]["us_above_empty_launch"] = above * 1e3
        rec["single"]["frac_above_empty_launch"] = (alg_bytes / (above * 1e-3) / 1e9 / hbm) if above > 0 else None
        rec["noalloc"] = noalloc_record(A, B, bias, C, cfg, alg_bytes, hbm, flush, dev, steps, warmup)
        rec["stream"] = decode_stream(A, bias, cfg, K, N, alg_bytes, hbm, flush, dev)
        rec["batched"] = decode_batched(A, bias, cfg, K, N, alg_bytes, hbm, flush, dev)
    else:
        rec["roofline"] = {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                           "algorithmic_bytes_per_launch": alg_bytes, "traffic": traffic,
                           "traffic_over_algorithmic": traffic / alg_bytes if traffic else None}
    rec["lean_pipeline_bound"] = lean_bound(rec["roofline"]["frac"], info["stages"])
    del A, B, bias, res, C
    torch.cuda.empty_cache()
    return rec


def noalloc_record(A, B, bias, C, cfg, alg_bytes, hbm, flush, dev, steps, warmup):
    """pax_gemm_skinny_noalloc on the same problem (its per-call counter
    clear included), timed like the single launch."""
    import torch

    import pax_b200

    d = pax_b200.make_desc(A, B, C, epilogue=cfg["epi"], bias=bias if "bias" in cfg["epi"] else None)
    lib = pax_b200.lib

    def step():
        st = lib.pax_gemm_skinny_noalloc(ctypes.byref(d), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
        if st != 0:
            raise RuntimeError(f"pax_gemm_skinny_noalloc: status {st}")

    r = timed_steps(step, steps, warmup, flush, dev, 1, dev.index)
    gbs = alg_bytes / (r["mean"] * 1e-3) / 1e9
    return {"us_per_gemm": r["mean"] * 1e3, "achieved": gbs, "frac": gbs / hbm,
            "note": "one GEMM launch, the layout pax_gemm_ex picks, scratch in a fixed device array "
                    "(no clearing: split-tile flags carry the launch epoch)"}


def split_record(args, dev, flush, peak, world, rank, local, steps, warmup, gather_too):
    """C5 (32768^3 BiasGeLU) strong-scaled: the N columns are split over the
    ranks, so total work is fixed as N grows.  Timed without replication
    and, at N > 1, with C replicated on every rank by the fused GEMM +
    all-gather (ReplicatedC)."""
    import torch

    import pax_b200
    from pax_b200.dist import ReplicatedC, slab_bounds

    cfg = CONFIGS[5]
    M, K, n_total = cfg["M"], cfg["K"], cfg["N"]
    s0, s1 = slab_bounds(n_total, world, rank)
    A, B, bias, _ = make_operands(cfg, M, s1 - s0, K, dev, args.seed, rank)
    C = torch.empty((M, s1 - s0), dtype=torch.float16, device=dev)
    flops = 2.0 * M * n_total * K
    r = timed_steps(lambda: pax_b200.gemm(A, B, out=C, epilogue=cfg["epi"], bias=bias), steps, warmup, flush, dev,
                    world, local)
    rec = {"workload": cfg["name"] + f", N split over {world} GPU(s) (strong scaling)", "steps": steps,
           "warmup": warmup, "ms_per_step": r["max_over_ranks"], "tflops_total": flops / (r["max_over_ranks"] * 1e-3) / 1e12,
           "clocks": r["clocks"]}
    rec["frac_of_peak_per_gpu"] = rec["tflops_total"] / world / peak
    rec["kernel"] = kernel_name(A, B, C, epilogue=cfg["epi"], bias=bias)
    del C
    if gather_too and world > 1:
        rc = ReplicatedC(M, n_total, device=dev)
        g = timed_steps(lambda: rc.gemm_slab(A, B, cfg["epi"], bias), steps, warmup, flush, dev, world, local)
        rec["replicated_fused"] = {"ms_per_step": g["max_over_ranks"],
                                   "tflops_total": flops / (g["max_over_ranks"] * 1e-3) / 1e12,
                                   "cost_vs_unreplicated": g["max_over_ranks"] / r["max_over_ranks"] - 1.0,
                                   "bytes_pushed_per_rank": M * (s1 - s0) * 2 * (world - 1),
                                   "ordering": rc.ordering}
        torch.cuda.synchronize()
        torch.distributed.barrier()
        rc.close()
        del rc
        if pax_b200.device_error() != pax_b200.Status.OK:
            raise RuntimeError("replicated C5: device-side wait timed out")
    del A, B, bias
    torch.cuda.empty_cache()
    return rec


def gather_record(A, B, bias, res, cfg, M, N, n_total, dev, flush, world, local, steps, warmup):
    """The C2 step with C replicated on every rank, three ways: the fused
    GEMM + all-gather (each finished tile copied to every peer's C over
    NVLink while later tiles compute), ordered by peer flag barriers or by
    two one-element NCCL all-reduces, and the GEMM followed by an NCCL
    all-gather of the slabs and a pack into row-major C."""
    import torch
    import torch.distributed as dist

    import pax_b200
    from pax_b200.dist import ReplicatedC, gather_columns

    flops = 2.0 * M * n_total * cfg["K"]
    kb = bias if "bias" in cfg["epi"] else None
    fused = {}
    for ordering in ("flags", "collective"):
        rc = ReplicatedC(M, n_total, device=dev, ordering=ordering)
        fused[ordering] = timed_steps(lambda: rc.gemm_slab(A, B, cfg["epi"], kb, res), steps, warmup, flush, dev,
                                      world, local)
        torch.cuda.synchronize()
        dist.barrier()
        rc.close()
        del rc
        if pax_b200.device_error() != pax_b200.Status.OK:
            raise RuntimeError(f"replicated C2 ({ordering} ordering): device-side wait timed out")
    f = fused["flags"]
    C = torch.empty((M, N), dtype=torch.float16, device=dev)

    def nccl_step():
        pax_b200.gemm(A, B, out=C, epilogue=cfg["epi"], bias=kb, residual=res)
        gather_columns(C)

    n = timed_steps(nccl_step, steps, warmup, flush, dev, world, local)
    torch.cuda.empty_cache()
    slab = M * N * 2
    c = fused["collective"]
    return {"fused": {"ms_per_step": f["max_over_ranks"], "tflops_total": flops / (f["max_over_ranks"] * 1e-3) / 1e12,
                      "how": "each finished tile TMA-copied from the local C to every peer's C over NVLink while "
                             "later tiles compute; a peer flag barrier (pax_peer_barrier) before and after"},
            "fused_nccl_ordering": {"ms_per_step": c["max_over_ranks"],
                                    "tflops_total": flops / (c["max_over_ranks"] * 1e-3) / 1e12,
                                    "how": "the same kernel, ordered by 2 one-element NCCL all-reduces"},
            "nccl": {"ms_per_step": n["max_over_ranks"], "tflops_total": flops / (n["max_over_ranks"] * 1e-3) / 1e12,
                     "how": "GEMM, then NCCL all_gather_into_tensor of the slabs and a pack into row-major C"},
            "bytes_per_rank_to_peers": slab * (world - 1)}


def run_pax(args):
    import numpy as np  # noqa: F401
    import torch
    import torch.distributed as dist

    import pax_b200

    rank, world, local = rank_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    cfg = config_for(args)
    from pax_b200.dist import ReplicatedC, equal_slabs, gather_columns, slab_bounds

    M, K = cfg["M"], cfg["K"]
    if args.strong:
        n_total = cfg["N"]
        s0, s1 = slab_bounds(n_total, world, rank)
        N = s1 - s0
    else:
        N = cfg["N"]
        n_total = N * world
    if args.gather and not (equal_slabs(n_total, world) or world == 1):
        raise SystemExit("--gather needs equal slabs (N divisible by 8 * ranks)")
    A, B, bias, res = make_operands(cfg, M, N, K, dev, args.seed, rank)
    C = torch.empty((M, N), dtype=torch.float16, device=dev)
    gathered = args.gather and world > 1
    flush = L2Flush(dev)
    kw = dict(epilogue=cfg["epi"], bias=bias if "bias" in cfg["epi"] else None, residual=res, out=C)

    rc = ReplicatedC(M, n_total, device=dev) if gathered and args.gather_impl == "fused" else None

    def step():
        if rc is not None:
            rc.gemm_slab(A, B, cfg["epi"], kw["bias"], res)
            return
        pax_b200.gemm(A, B, **kw)
        if gathered:
            gather_columns(C)

    main = timed_steps(step, args.steps, args.warmup, flush, dev, world, local)
    ms = main["ms"]
    ms_max = main["max_over_ranks"]
    clk = main["clocks"]
    flops_rank = 2.0 * M * N * K
    flops_total = 2.0 * M * n_total * K
    value = flops_total / (ms_max * 1e-3) / 1e12

    # ---- end to end through the public API: pinned host inputs, host output.
    # Steps alternate between two streams with their own device and host
    # buffers, as a serving loop would run them: each step still uploads its
    # inputs, runs the GEMM and reads C back, but one step's upload overlaps
    # the previous step's GEMM and download (PCIe is full duplex).
    hA = A.cpu().pin_memory()
    hB = B.cpu().pin_memory()
    hbias = bias.cpu().pin_memory()
    hres = res.cpu().pin_memory() if res is not None else None
    h2d = hA.numel() * 2 + hB.numel() * 2 + (hbias.numel() * 2 if "bias" in cfg["epi"] else 0) + (
        hres.numel() * 2 if hres is not None else 0)
    d2h = M * N * 2
    slots = []
    for _ in range(2):
        slots.append(dict(stream=torch.cuda.Stream(device=dev), A=torch.empty_like(A), B=torch.empty_like(B),
                          bias=torch.empty_like(bias), res=torch.empty_like(res) if res is not None else None,
                          C=torch.empty((M, N), dtype=torch.float16, device=dev),
                          hC=torch.empty((M, N), dtype=torch.float16).pin_memory()))

    def e2e_step(i):
        sl = slots[i % 2]
        with torch.cuda.stream(sl["stream"]):
            sl["A"].copy_(hA, non_blocking=True)
            sl["B"].copy_(hB, non_blocking=True)
            if "bias" in cfg["epi"]:
                sl["bias"].copy_(hbias, non_blocking=True)
            if sl["res"] is not None:
                sl["res"].copy_(hres, non_blocking=True)
            pax_b200.gemm(sl["A"], sl["B"], epilogue=cfg["epi"], bias=sl["bias"] if "bias" in cfg["epi"] else None,
                          residual=sl["res"], out=sl["C"])
            sl["hC"].copy_(sl["C"], non_blocking=True)

    e2e_steps = max(4, min(args.steps, 10))
    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    cur = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for sl in slots:
        sl["stream"].wait_stream(cur)
    for i in range(e2e_steps):
        e2e_step(i)
    for sl in slots:
        cur.wait_stream(sl["stream"])
    e1.record(cur)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = flops_total / (float(t.item()) * 1e-3) / 1e12
    del slots, hA, hB, hbias, hres

    peak, hbm, peak_kind = peaks()
    stages = pax_b200.pipeline_stages(A, B, C, epilogue=cfg["epi"], bias=bias if "bias" in cfg["epi"] else None,
                                      residual=res)
    kernel_ms = None if gathered else min(ms)
    achieved = None if gathered else flops_rank / (statistics.mean(ms) * 1e-3) / 1e12
    roofline = None
    if achieved is not None:
        alg_bytes = 2 * (M * K + K * N + M * N) + (2 * N if "bias" in cfg["epi"] else 0) + (
            2 * M * N if res is not None else 0)
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "traffic": traffic_from_profiles(args.config),
                    "peak_kind": f"{peak_kind} (bf16 dense burst, MEASURED_PEAKS.json)" if peak_kind == "measured"
                    else "fallback 1.59 PFLOP/s", "algorithmic_flops_per_launch": flops_rank,
                    "algorithmic_bytes_per_launch": alg_bytes, "best_launch_ms": kernel_ms}
        if args.config == 4:
            gbs = alg_bytes / (statistics.mean(ms) * 1e-3) / 1e9
            roofline = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                        "traffic": traffic_from_profiles(args.config),
                        "peak_kind": f"{peak_kind} (copy bandwidth)", "algorithmic_bytes_per_launch": alg_bytes,
                        "tflops": achieved, "best_launch_ms": kernel_ms,
                        "stream": decode_stream(A, bias, cfg, K, N, alg_bytes, hbm, flush, dev),
                        "batched": decode_batched(A, bias, cfg, K, N, alg_bytes, hbm, flush, dev)}
        if roofline["traffic"]:
            roofline["traffic_over_algorithmic"] = roofline["traffic"] / alg_bytes

    # ---- sub-records.  At N = 1 the other four configurations, each device-
    # timed like the headline; at N > 1 the collective: the same step with C
    # replicated (fused and NCCL), and C5 split over the ranks.
    sub = {}
    defaults = args.config == 2 and not args.epilogue and args.m is None and not args.strong and not args.gather

    def guarded(name, fn):
        """Run one sub-record; an error is recorded in the line instead of
        losing the headline.  Every rank takes the same steps, and the ranks
        agree (one all-reduce) on whether all of them succeeded, so that none
        goes on into later collectives alone."""
        try:
            out, ok = fn(), 1
        except Exception as e:  # noqa: BLE001 - reported in the JSON line
            out, ok = {"error": f"{type(e).__name__}: {e}"[:300]}, 0
        if world > 1:
            t = torch.tensor([ok], dtype=torch.int32, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            ok = int(t.item())
        torch.cuda.empty_cache()
        return out, ok == 1

    if defaults and not args.no_subrecords:
        ok = True
        if world == 1:
            sub["configs"] = {}
            for cid, st, wu in ((1, args.steps, max(3, args.warmup)), (3, min(args.steps, 20), max(3, args.warmup)),
                                (4, args.steps, max(3, args.warmup))):
                sub["configs"][f"C{cid}"], _ = guarded(
                    f"C{cid}", lambda cid=cid, st=st, wu=wu: config_record(cid, args, dev, flush, peak, hbm, st, wu))
        else:
            sub["gather"], ok = guarded("gather", lambda: gather_record(
                A, B, bias, res, cfg, M, N, n_total, dev, flush, world, local, min(args.steps, 20),
                max(3, args.warmup)))
        if ok:
            # C5 over the ranks: 55 ms per launch on one GPU, so a few steps.
            c5, _ = guarded("c5", lambda: split_record(args, dev, flush, peak, world, rank, local, 3, 3,
                                                       gather_too=True))
            if world == 1:
                if "tflops_total" in c5:
                    a = c5["tflops_total"]
                    c5["roofline"] = {"bound": "tensor", "achieved": a, "peak": peak, "unit": "TFLOP/s",
                                      "frac": a / peak, "traffic": traffic_from_profiles(5)}
                    c5["lean_pipeline_bound"] = lean_bound(a / peak, c5["kernel"]["stages"])
                sub["configs"]["C5"] = c5
            else:
                sub["c5_split"] = c5

    # Clocks over a long back-to-back run of the headline step: enough NVML
    # samples to say what SM clock the kernel runs at under sustained load.
    if defaults and world == 1 and not args.no_subrecords:
        sub["sustained"], _ = guarded("sustained", lambda: sustained_record(step, dev, local, flops_rank))
        sub["same_box_comparison"], _ = guarded("same_box_comparison", lambda: comparison_record(
            A, B, C, dev, flush, flops_rank, args.steps, max(3, args.warmup)))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, dt, rows, threads, kind, _ = cpu_gemm_sample(cfg, args.cpu_seconds, args.seed)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": kind,
               "sample": f"{rows} of {M} rows of the same GEMM (cpu_gemm_ref i-j-l fp32 loop) in {dt:.1f} s on "
                         f"{threads} host threads"}
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_max,
            "higher_is_better": True,
            "scaling": "strong" if args.strong else "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (seeded torch RNG on device: " + (
                "A,B uniform[-1,1]" if cfg["dist"] == "uniform" else "A N(0,1), B N(0,0.02)") + ", bias N(0,1))",
            "config": workload_config(cfg, world, args),
            "pct_of_dense_fp16_peak": 100.0 * (value / world) / peak,
            "gemm_ms_per_rank": ms_max,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "pipelining": "steps alternate between 2 streams (each step: upload inputs, GEMM, download C)"},
            "clocks": clk,
            "gpu_launches": args.steps,
            "lean_pipeline_bound": lean_bound(roofline["frac"] if roofline else None, stages),
        }
        line.update(sub)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        if rc is not None:
            rc.close()
        dist.destroy_process_group()
    return 0


def comparison_record(A, B, C, dev, flush, flops, steps, warmup):
    """The headline shape without its epilogue, this library's kernel and
    cuBLAS (torch.matmul, fp16), timed like the headline on the same GPU:
    the speed of each GEMM alone, since clocks differ from box to box."""
    import torch

    import pax_b200

    ours = timed_steps(lambda: pax_b200.gemm(A, B, out=C), steps, warmup, flush, dev, 1, dev.index)
    lib = timed_steps(lambda: torch.matmul(A, B, out=C), steps, warmup, flush, dev, 1, dev.index)
    return {"pax_no_epilogue": {"ms_per_launch": ours["mean"], "tflops": flops / (ours["mean"] * 1e-3) / 1e12},
            "cublas_no_epilogue": {"ms_per_launch": lib["mean"], "tflops": flops / (lib["mean"] * 1e-3) / 1e12,
                                   "how": "torch.matmul fp16 (cuBLAS), same operands, L2 flush and event timing"}}


def sustained_record(step, dev, local, flops, seconds=0.25):
    """The headline step back to back (no L2 flush) for about `seconds`,
    with NVML clock samples throughout: mean ms per launch, the median SM
    clock under this load and their product, the cycles one launch takes."""
    import torch

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(5):
        step()
    torch.cuda.synchronize()
    per = max((time.perf_counter() - t0) / 5, 1e-5)
    n = int(min(20000, max(50, seconds / per)))
    clocks = clock_sampler(local)
    clocks.start()
    time.sleep(0.2)
    anchor = torch.cuda.Event(enable_timing=True)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    anchor.record()
    t_anchor = time.perf_counter()
    torch.cuda._sleep(int(0.05 * 2.0e9))
    e0.record()
    for _ in range(n):
        step()
    e1.record()
    torch.cuda.synchronize()
    window = (t_anchor + anchor.elapsed_time(e0) * 1e-3, t_anchor + anchor.elapsed_time(e1) * 1e-3)
    clk = clocks.stop(window) if isinstance(clocks, NvmlSampler) else clocks.stop()
    ms = e0.elapsed_time(e1) / n
    rec = {"launches": n, "ms_per_launch": ms, "tflops": flops / (ms * 1e-3) / 1e12, "clocks": clk,
           "note": "back to back, no L2 flush; same kernel and problem as the headline"}
    if clk is not None:
        rec["kcycles_per_launch_at_median_mhz"] = ms * clk["sm_mhz"]
    return rec


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    return run_pax(args)


if __name__ == "__main__":
    sys.exit(main())
