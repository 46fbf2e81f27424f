#!/usr/bin/env python
"""Benchmark of the wavelet filter-bank hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config cfg2]

Default workload (configs[1] of the baseline, the one the headline metric is quoted on):
db8 ``periodization`` level-8 ``wavedec`` of x float32 (16, 128, 65536) i.i.d. N(0,1), ``waverec``
of the coefficients, and the autograd backward through both.  One step = those four
multilevel transforms over the whole batch (each a chain of streaming launches, two levels
per launch where the shapes allow);
inputs (512 MiB per array) are larger than the 126 MB L2.

``value`` is the whole-job algorithmic HBM throughput in GB/s (unique bytes the four transforms
must read and write: inputs once, outputs once), device-timed with CUDA events over K steps,
max over ranks.  Each rank runs the full config on its own data ("weak" scaling: the path
shards by rows and has no collective).  ``e2e`` repeats the step through the public API with
the input in pinned host memory and the gradient copied back every step.

``--impl reference`` times the reference algorithm's CPU path (the oracle port in ``oracle/``,
restating the reference's own CPU code) on the host cores, on a bounded row sample per step.
"""

from __future__ import annotations

import argparse
import json
import math
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "DWT/CWT achieved HBM GB/s (% of B200 peak); Morlet mixer tokens/s fwd+bwd"
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) per full-size launch of the kernels of the two finest levels, from
# one ncu capture of each on 1024 of the 2048 rows scaled by 2 (traffic grows with the rows);
# the captures are summarised in profiles/dwt_cfg2_kernels.txt
TRAFFIC_PER_LAUNCH = {
    "dwt_ana2_stream_kernel<float,16>": 974_800_000,
    "dwt_syn2_stream_kernel<float,16,0>": 970_000_000,
}


# ------------------------------------------------------------------------------ helpers

def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """SM clock and clock-event reasons of this rank's GPU, sampled through NVML (read only)
    every few milliseconds by a background thread while the timed region runs."""

    def __init__(self, device_index: int, period_s: float = 0.004):
        self.index = device_index
        self.period = period_s
        self.samples, self.reasons, self.smax = [], set(), None
        self.handle = None
        self.thread = None
        self.stop = threading.Event()

    def _open(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.index)
        uuid = getattr(props, "uuid", None)
        if uuid is not None:
            try:
                return pynvml, pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{uuid}")
            except pynvml.NVMLError:
                pass
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)

    def _run(self, nv):
        bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap,
                "hw_power_brake": nv.nvmlClocksEventReasonHwPowerBrakeSlowdown}
        while not self.stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.reasons.update(k for k, b in bits.items() if r & b)
            except nv.NVMLError:
                break
            time.sleep(self.period)

    def __enter__(self):
        try:
            nv, self.handle = self._open()
            self.smax = nv.nvmlDeviceGetMaxClockInfo(self.handle, nv.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._run, args=(nv,), daemon=True)
            self.thread.start()
        except Exception:  # no NVML: reported as unsampled
            self.thread = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.smax, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.smax,
                "samples": len(self.samples), "reasons": sorted(self.reasons)}


def max_over_ranks(values, world, device):
    """Element-wise maximum of per-rank timings over all ranks (identity for one rank)."""
    import torch
    t = torch.tensor([float(v) for v in values], device=device, dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.cpu()]


def job_throughput(units_per_rank_step, steps, world, ms, scale=1.0):
    """Whole-job rate: the units every rank processed over the slowest rank's time."""
    return units_per_rank_step * steps * world / (ms / 1e3) / scale


# ------------------------------------------------------------------------------ workload

CFG2 = dict(shape=(16, 128, 65536), wavelet="db8", mode="periodization", level=8)


def cfg2_bytes_per_row():
    """Algorithmic bytes of one row through the four launches of a step (fp32)."""
    from oracle.dwt_oracle import dwt_coeff_len
    n = CFG2["shape"][-1]
    lens, cur = [], n
    for _ in range(CFG2["level"]):
        cur = dwt_coeff_len(cur, 16, CFG2["mode"])
        lens.append(cur)
    coef = sum(lens) + lens[-1]
    per_dir = (n + coef) * 4  # read one side, write the other
    return 4 * per_dir, per_dir


def _cpu_rows_task(args):
    """One worker: the full step on a chunk of rows, with the oracle (fp32)."""
    rows, seed = args
    from oracle import dwt_oracle as D
    from pytorch_morlet_fdwt_b200.wavelets import get_filter_bank
    b = get_filter_bank(CFG2["wavelet"])
    tb = (b.dec_lo, b.dec_hi, b.rec_lo, b.rec_hi)
    x = np.random.default_rng(seed).standard_normal((rows, CFG2["shape"][-1])).astype(np.float32)
    t = time.perf_counter()
    c = D.wavedec(x, tb, CFG2["mode"], CFG2["level"])
    y = D.waverec(c, tb, CFG2["mode"])
    gc = D.waverec_vjp(c, y, tb, CFG2["mode"])
    D.wavedec_vjp(x.shape[-1], gc, tb, CFG2["mode"])
    return time.perf_counter() - t


class CpuPool:
    """Spawned worker pool for the CPU oracle (created before any CUDA call)."""

    def __init__(self, cores: int):
        self.cores = cores
        self.pool = mp.get_context("spawn").Pool(cores)
        self.pool.map(_cpu_rows_task, [(2, 0)] * cores)  # import + operator caches warm

    def step(self, rows: int) -> float:
        per = max(1, rows // self.cores)
        t = time.perf_counter()
        self.pool.map(_cpu_rows_task, [(per, i) for i in range(self.cores)])
        return time.perf_counter() - t, per * self.cores

    def close(self):
        self.pool.close()
        self.pool.join()


def cpu_sample(pool: CpuPool, rows: int, reps: int):
    times = []
    done = rows
    for _ in range(reps):
        t, done = pool.step(rows)
        times.append(t)
    t = statistics.median(times)
    step_bytes, _ = cfg2_bytes_per_row()
    return step_bytes * done / t / 1e9, t, done


# ------------------------------------------------------------------------------ our arm

def run_ours(args, rank, world, local_rank, pool):
    import torch
    import torch.distributed as dist
    import pytorch_morlet_fdwt_b200 as F
    from pytorch_morlet_fdwt_b200 import _lib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    torch.manual_seed(1234 + rank)
    shape = CFG2["shape"]
    if args.rows is not None:
        shape = (1, args.rows, shape[-1])
    bank = F.get_filter_bank(CFG2["wavelet"])
    mode, level = CFG2["mode"], CFG2["level"]
    x0 = torch.randn(shape, device=dev)
    R = shape[0] * shape[1]
    step_bytes_row, dir_bytes_row = cfg2_bytes_per_row()
    step_bytes = step_bytes_row * R
    gy = torch.randn(shape, device=dev)

    def step(x):
        coeffs = F.wavedec(x, bank, mode, level)
        y = F.waverec(coeffs, bank, mode)
        torch.autograd.backward(y, gy)

    def barrier():
        if world > 1:
            dist.barrier()

    x = x0.clone().requires_grad_()
    for _ in range(args.warmup):
        x.grad = None
        step(x)
    torch.cuda.synchronize()

    # device time of the two multilevel calls of the step (wavedec; also the waverec backward,
    # and waverec; also the wavedec backward), each timed on its forward call
    ka, kb, kc = ([torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
                  for _ in range(3))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _lib.launch_count()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        start.record()
        for i in range(args.steps):
            x.grad = None
            ka[i].record()
            coeffs = F.wavedec(x, bank, mode, level)
            kb[i].record()
            y = F.waverec(coeffs, bank, mode)
            kc[i].record()
            torch.autograd.backward(y, gy)
        end.record()
        torch.cuda.synchronize()
    barrier()
    launches = _lib.launch_count() - launches0
    ms = start.elapsed_time(end)
    ana_ms = statistics.mean(a.elapsed_time(b) for a, b in zip(ka, kb))
    syn_ms = statistics.mean(b.elapsed_time(c) for b, c in zip(kb, kc))
    ms, ana_ms, syn_ms = max_over_ranks([ms, ana_ms, syn_ms], world, dev)
    kernels = finest_launch_ms(F, _lib, x0, bank, mode, max(3, args.steps), barrier)
    vals = max_over_ranks(list(kernels.values()), world, dev)
    kernels = dict(zip(kernels, vals))

    # end to end through the public API with host buffers (pinned), every step
    e2e_steps = max(1, min(args.steps, 10))
    e2e_ms = float("nan")
    if args.no_e2e:
        return _finish_cfg2(args, rank, world, R, step_bytes, dir_bytes_row, ms, ana_ms, syn_ms,
                            kernels, launches, clk, pool, x0, e2e_steps, e2e_ms, shape)
    e2e_ms = e2e_pipelined(step, x0, e2e_steps, max(1, args.warmup // 2), barrier)
    (e2e_ms,) = max_over_ranks([e2e_ms], world, dev)
    return _finish_cfg2(args, rank, world, R, step_bytes, dir_bytes_row, ms, ana_ms, syn_ms,
                        kernels, launches, clk, pool, x0, e2e_steps, e2e_ms, shape)


def e2e_pipelined(step, x0, steps, warmup, barrier):
    """Device time of `steps` end-to-end steps: every step copies its input from pinned host
    memory (host->device), runs the step through the public API and copies the result (the
    input gradient, as large as the input) back to pinned host memory.  The copies run on
    their own streams, double-buffered, so that step i+1's upload and step i's download overlap
    step i's kernels and each other (PCIe is full duplex); the timed region runs from the first
    upload to the last download."""
    import torch
    dev = x0.device
    xh = x0.cpu().pin_memory()
    gh = [torch.empty_like(xh).pin_memory() for _ in range(2)]
    xd = [torch.empty_like(x0) for _ in range(2)]
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event(enable_timing=False)

    def run(n, timed):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        uploaded = [ev() for _ in range(n)]
        consumed = [None, None]   # compute done with xd[b]
        computed = [ev() for _ in range(n)]
        downloaded = [None, None]  # gh[b] and the gradient of the step that used b are free
        grads = [None, None]
        if timed:
            start.record(s_in)
        for i in range(n):
            b = i % 2
            with torch.cuda.stream(s_in):
                if consumed[b] is not None:
                    s_in.wait_event(consumed[b])
                xd[b].copy_(xh, non_blocking=True)
                uploaded[i].record(s_in)
            comp.wait_event(uploaded[i])
            if downloaded[b] is not None:
                comp.wait_event(downloaded[b])
            xe = xd[b].detach().requires_grad_()
            step(xe)
            grads[b] = xe.grad
            consumed[b] = ev()
            consumed[b].record(comp)
            computed[i].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(computed[i])
                gh[b].copy_(grads[b], non_blocking=True)
                downloaded[b] = ev()
                downloaded[b].record(s_out)
        if timed:
            end.record(s_out)
        torch.cuda.synchronize()
        return start.elapsed_time(end) if timed else 0.0

    run(warmup, False)
    barrier()
    torch.cuda.synchronize()
    return run(steps, True)


def finest_launch_ms(F, _lib, x0, bank, mode, reps, barrier):
    """Device time of one launch of each dominant kernel: the two finest levels of the analysis
    (a two-level wavedec of the whole batch: one dwt_ana2_stream_kernel launch) and of the
    synthesis (a two-level waverec: one dwt_syn2_stream_kernel launch), each the largest launch
    of its direction in the step.  Timed with CUDA events around `reps` back-to-back calls
    (each call must be one launch)."""
    import torch
    x2 = x0.reshape(-1, x0.shape[-1])
    c2 = F.wavedec(x2, bank, mode, 2)
    out = {}
    for name, fn in (("dwt_ana2_stream_kernel<float,16>", lambda: F.wavedec(x2, bank, mode, 2)),
                     ("dwt_syn2_stream_kernel<float,16,0>", lambda: F.waverec(c2, bank, mode))):
        for _ in range(2):
            fn()
        barrier()
        torch.cuda.synchronize()
        l0 = _lib.launch_count()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        if _lib.launch_count() - l0 != reps:
            raise RuntimeError(f"{name}: a two-level call was not exactly one launch")
        out[name] = e0.elapsed_time(e1) / reps
    return out


def _finish_cfg2(args, rank, world, R, step_bytes, dir_bytes_row, ms, ana_ms, syn_ms, kernels,
                 launches, clk, pool, x0, e2e_steps, e2e_ms, shape):
    if rank != 0:
        return None
    peak, peak_src = peaks()
    value = job_throughput(step_bytes, args.steps, world, ms, 1e9)
    dominant = max(kernels, key=kernels.get)
    kern_ms = kernels[dominant]
    achieved = dir_bytes_row * R / (kern_ms / 1e3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic i.i.d. N(0,1), seeded per rank",
        "config": {
            "workload": "cfg2: db8 periodization level-8 wavedec + waverec + backward through "
                        f"both, x float32 {tuple(shape)} per GPU",
            "algorithmic_bytes_per_step": step_bytes,
            "l2": "inputs larger than L2 (512 MiB per array)",
            "parallelism": f"rows sharded by rank, {world} GPU(s), no collective",
        },
        "roofline": {
            "bound": "hbm", "kernel": dominant,
            "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": peak_src,
            "algorithmic_bytes_per_launch": dir_bytes_row * R,
            "launch_ms": round(kern_ms, 4),
            "traffic": TRAFFIC_PER_LAUNCH.get(dominant),
            "kernels_ms_per_launch": {k: round(v, 4) for k, v in kernels.items()},
            "launch": "the two finest levels of the step's analysis / synthesis in one launch "
                      "over every row: x (or the level-1 details and level-2 coefficients) "
                      "read once, the other side written once",
            "calls_ms": {"wavedec (8 levels, 4 launches)": round(ana_ms, 4),
                         "waverec (8 levels, 4 launches)": round(syn_ms, 4)},
        },
        "gpu_launches": int(launches),
        "e2e": None if args.no_e2e else {
            "value": round(step_bytes * e2e_steps * world / (e2e_ms / 1e3) / 1e9, 2),
            "unit": "GB/s",
            "h2d_bytes_per_step": x0.numel() * 4,
            "d2h_bytes_per_step": x0.numel() * 4,
            "ms_per_step": round(e2e_ms / e2e_steps, 3),
            "copies": "input upload and gradient download of every step on their own streams, "
                      "double-buffered: step i+1's upload and step i's download overlap step "
                      "i's kernels",
        },
        "clocks": clk.summary(),
    }
    if pool is not None:
        gbs, t, rows = cpu_sample(pool, rows=args.cpu_rows, reps=3)
        line["cpu_baseline"] = {
            "value": round(gbs, 3), "unit": "GB/s", "cores": pool.cores, "kind": "port",
            "sample": f"{rows} of the 2048 rows of the cfg2 step (wavedec, waverec, both "
                      f"vjps) with the oracle's sparse-operator restatement in fp32, median of 3 "
                      f"({t:.2f} s each)",
        }
    return line


# ------------------------------------------------------------------------------ reference arm

def run_reference(args, pool):
    times = []
    rows_done = 0
    for i in range(args.warmup + args.steps):
        t, rows_done = pool.step(args.cpu_rows)
        if i >= args.warmup:
            times.append(t)
    step_bytes_row, _ = cfg2_bytes_per_row()
    t = statistics.mean(times)
    value = step_bytes_row * rows_done / t / 1e9
    sample = (f"{rows_done} rows of the cfg2 step per step (wavedec, waverec, both vjps) with the "
              f"oracle port of the reference's CPU path, fp32, {pool.cores} worker processes")
    return {
        "metric": METRIC, "impl": "reference", "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic i.i.d. N(0,1)",
        "config": {"workload": "cfg2: db8 periodization level-8 wavedec + waverec + backward "
                               "through both (bounded row sample of (16,128,65536))"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": pool.cores,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------------------ other configs
#
# The other baseline configs (2, 3, 4), measured the same way on demand with
# --config; each prints its own line.  The forward and the backward calls are timed separately
# with CUDA events; the kernel named in "roofline" is the one with the larger share.


def _cfg_cwt_plan(learnable):
    import pytorch_morlet_fdwt_b200 as F
    return F.CWT1D(freqs=np.logspace(-0.3, 2, 40), fs=250.0, norm="l1", learnable=learnable,
                   learnable_w0=learnable)


def _wl_cfg1():
    import torch
    import pytorch_morlet_fdwt_b200 as F
    from oracle.dwt_oracle import dwt_coeff_len
    n, lv = 2500, 5
    lens, cur = [], n
    for _ in range(lv):
        cur = dwt_coeff_len(cur, 8, "symmetric")
        lens.append(cur)
    rows = 32 * 64
    per_dir = rows * (n + sum(lens) + lens[-1]) * 4

    def setup(dev):
        return {"x": torch.randn(32, 64, n, device=dev).requires_grad_(),
                "bank": F.get_filter_bank("db4")}

    def fwd(st):
        st["c"] = F.wavedec(st["x"], st["bank"], "symmetric", lv)
        st["y"] = F.waverec([c.detach() for c in st["c"]], st["bank"], "symmetric")

    def bwd(st):
        st["x"].grad = None
        sum((c * c).sum() for c in st["c"]).backward()

    def cpu(rows_s):
        from oracle import dwt_oracle as D
        b = F.get_filter_bank("db4")
        tb = (b.dec_lo, b.dec_hi, b.rec_lo, b.rec_hi)
        x = np.random.default_rng(0).standard_normal((rows_s, n)).astype(np.float32)
        t = time.perf_counter()
        c = D.wavedec(x, tb, "symmetric", lv)
        D.waverec(c, tb, "symmetric")
        D.wavedec_vjp(n, [2 * v for v in c], tb, "symmetric")
        return time.perf_counter() - t

    return dict(name="cfg1: db4 symmetric level-5 wavedec, waverec and the backward of "
                     "sum(coeffs^2), x float32 (32,64,2500)",
                unit="GB/s", per_step=3 * per_dir, rows=rows, setup=setup, fwd=fwd, bwd=bwd,
                cpu=cpu, cpu_rows=2048, dtype="f32",
                kernels=("dwt_analysis_kernel + dwt_syn_tile_kernel (waverec)",
                         "dwt_syn_tile_kernel (backward)"),
                fwd_bytes=2 * per_dir, bwd_bytes=per_dir)


def _wl_cfg3(learnable, rows=None):
    import torch
    from oracle import cwt_oracle as C
    shape = (32 if rows is None else max(1, rows // 64), 64, 2500)
    rows = shape[0] * shape[1]
    x_bytes = rows * 2500 * 4
    w_bytes = rows * 40 * 2500 * 8

    def setup(dev):
        m = _cfg_cwt_plan(learnable).to(dev)
        return {"m": m, "x": torch.randn(shape, device=dev).requires_grad_(learnable)}

    def fwd(st):
        st["y"] = st["m"](st["x"])

    def bwd(st):
        if learnable:
            st["x"].grad = None
            st["m"].zero_grad()
            torch.view_as_real(st["y"]).square().sum().backward()

    def cpu(rows_s):
        m = _cfg_cwt_plan(learnable)
        po = C.Plan(m.plan.scales, norm="l1", support_margin=1.25 if learnable else 1.0)
        ls = torch.tensor(m.plan.scales, dtype=torch.float64).log().requires_grad_(learnable)
        w0 = torch.tensor(6.0, dtype=torch.float64, requires_grad=learnable)
        x = torch.randn(rows_s, 2500, dtype=torch.float64, requires_grad=learnable)
        t = time.perf_counter()
        W = C.apply_plan(x, po, po.filters(ls.exp(), w0))
        if learnable:
            W.abs().square().sum().backward()
        return time.perf_counter() - t

    fb = x_bytes + w_bytes
    bb = w_bytes + 2 * x_bytes if learnable else 0
    name = ("cfg3: Morlet CWT fast, 40 freqs logspace(-0.3,2) @ 250 Hz, l1, x float32 "
            f"{shape} -> complex64 ({shape[0]},64,40,2500)")
    if learnable:
        name += "; learnable scales and w0, backward of sum |W|^2"
    return dict(name=name, unit="GB/s", per_step=fb + bb, rows=rows, setup=setup, fwd=fwd,
                bwd=bwd, cpu=cpu, cpu_rows=32 if learnable else 64, dtype="f32",
                kernels=("cwt_forward_kernel<float,float,0>", "cwt_backward_kernel<float,0>"),
                fwd_bytes=fb, bwd_bytes=bb)


def _wl_cfg4():
    import torch
    import pytorch_morlet_fdwt_b200 as F
    from oracle import cwt_oracle as C
    freqs = np.logspace(0, 1.8, 16).tolist()

    def setup(dev):
        torch.manual_seed(0)
        m = F.MorletTokenMixer(256, freqs=freqs, fs=250).to(dev)
        return {"m": m, "x": torch.randn(8, 4096, 256, device=dev).requires_grad_()}

    def fwd(st):
        st["y"] = st["m"](st["x"])

    def bwd(st):
        st["x"].grad = None
        st["m"].zero_grad()
        st["y"].square().sum().backward()

    def cpu(batch):
        torch.manual_seed(0)
        m = F.MorletTokenMixer(256, freqs=freqs, fs=250).double()
        po = C.Plan(m.cwt.plan.scales, support_margin=1.25)
        x = torch.randn(batch, 4096, 256, dtype=torch.float64, requires_grad=True)
        ls = m.cwt.log_scales.detach().double().requires_grad_()
        t = time.perf_counter()
        y = C.token_mixer(x, po, po.filters(ls.exp(), m.cwt.w0_value), m.mag_weight,
                          m.phase_weight, m.bias, m.out_proj.weight, m.out_proj.bias)
        y.square().sum().backward()
        return time.perf_counter() - t

    return dict(name="cfg4: MorletTokenMixer dim 256, 16 freqs logspace(0,1.8) @ 250 Hz, "
                     "x float32 (8,4096,256), forward + backward",
                unit="tokens/s", per_step=8 * 4096, rows=8 * 256, setup=setup, fwd=fwd, bwd=bwd,
                cpu=cpu, cpu_rows=1, cpu_unit_per_row=4096, cpu_reps=1, dtype="f32",
                kernels=("cwt_forward_kernel<float,float,1> (mix)",
                         "cwt_backward_kernel<float,1> (mix)"),
                fwd_bytes=2 * 8 * 4096 * 256 * 4, bwd_bytes=3 * 8 * 4096 * 256 * 4)


def _wl_cfg5(channel_mix):
    import torch
    import pytorch_morlet_fdwt_b200 as F
    from oracle import cwt_oracle as C
    cls = F.MorletChannelMixAttention if channel_mix else F.MorletAttention

    def setup(dev):
        torch.manual_seed(0)
        m = cls(num_channels=19, hidden_dim=200).to(dev)
        return {"m": m, "x": torch.randn(64, 4, 19, 30, 200, device=dev).requires_grad_()}

    def fwd(st):
        st["y"] = st["m"](st["x"])

    def bwd(st):
        st["x"].grad = None
        st["m"].zero_grad()
        st["y"].square().sum().backward()

    def cpu(batch):
        torch.manual_seed(0)
        m = cls(num_channels=19, hidden_dim=200).double()
        po = C.Plan(m.cwt.plan.scales, support_margin=1.25)
        x = torch.randn(batch, 4, 19, 30, 200, dtype=torch.float64, requires_grad=True)
        ls = m.cwt.log_scales.detach().double().requires_grad_()
        w0 = torch.tensor(m.cwt.w0_value, dtype=torch.float64, requires_grad=True)
        H = po.filters(ls.exp(), w0)
        t = time.perf_counter()
        if channel_mix:
            y = C.channel_mix_attention(x, po, H, m.freq_to_channel, m.temperature)
        else:
            y = C.attention(x, po, H, m.freq_weight, m.temperature)
        y.square().sum().backward()
        return time.perf_counter() - t

    name = ("cfg5: Morlet" + ("ChannelMix" if channel_mix else "") + "Attention, 19 channels, "
            "hidden 200, x float32 (64,4,19,30,200), forward + backward")
    return dict(name=name, unit="tokens/s", per_step=64 * 19 * 30, rows=64 * 4 * 19,
                setup=setup, fwd=fwd, bwd=bwd, cpu=cpu, cpu_rows=1, cpu_unit_per_row=19 * 30,
                dtype="f32",
                kernels=("cwt_forward_kernel<float,float,2> (spectral softmax)",
                         "cwt_backward_kernel<float,2> (spectral softmax)"),
                fwd_bytes=2 * 64 * 4 * 19 * 6000 * 4, bwd_bytes=3 * 64 * 4 * 19 * 6000 * 4)


WORKLOADS = {
    "cfg1": _wl_cfg1,
    "cfg3": lambda rows=None: _wl_cfg3(False, rows),
    "cfg3l": lambda rows=None: _wl_cfg3(True, rows),
    "cfg4": _wl_cfg4,
    "cfg5": lambda: _wl_cfg5(False),
    "cfg5c": lambda: _wl_cfg5(True),
}


def run_config(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from pytorch_morlet_fdwt_b200 import _lib
    W = WORKLOADS[args.config](args.rows) if args.rows else WORKLOADS[args.config]()
    # CPU baseline first (before any CUDA work), rank 0 at N=1
    cpu_line = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import torch as _t
        _t.set_num_threads(os.cpu_count() or 1)
        reps = W.get("cpu_reps", 3)
        if reps > 1:
            W["cpu"](W["cpu_rows"])  # warm-up
        times = [W["cpu"](W["cpu_rows"]) for _ in range(reps)]
        tc = statistics.median(times)
        units = W.get("cpu_unit_per_row")
        per = (W["cpu_rows"] * units) if units else W["per_step"] * W["cpu_rows"] / W["rows"]
        cpu_line = {"value": round(per / tc / (1e9 if W["unit"] == "GB/s" else 1), 4),
                    "unit": W["unit"], "cores": os.cpu_count(), "kind": "port",
                    "sample": f"{W['cpu_rows']} {'batch entries' if units else 'rows'} of the "
                              f"workload through the fp64 CPU oracle (torch, all cores), median "
                              f"of {reps} ({tc:.2f} s each)"}
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    torch.manual_seed(100 + rank)
    st = W["setup"](dev)
    for _ in range(args.warmup):
        W["fwd"](st)
        W["bwd"](st)
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    l0 = _lib.launch_count()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        for e in ev:
            e[0].record()
            W["fwd"](st)
            e[1].record()
            W["bwd"](st)
            e[2].record()
        torch.cuda.synchronize()
    launches = _lib.launch_count() - l0
    ms = ev[0][0].elapsed_time(ev[-1][2])
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    ms, fwd_ms, bwd_ms = max_over_ranks([ms, fwd_ms, bwd_ms], world, dev)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    scale = 1e9 if W["unit"] == "GB/s" else 1.0
    value = job_throughput(W["per_step"], args.steps, world, ms, scale)
    peak, peak_src = peaks()
    dom = 0 if fwd_ms >= bwd_ms or W["bwd_bytes"] == 0 else 1
    k_ms = fwd_ms if dom == 0 else bwd_ms
    k_bytes = W["fwd_bytes"] if dom == 0 else W["bwd_bytes"]
    achieved = k_bytes / (k_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": W["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": W["dtype"],
        "data": "synthetic i.i.d. N(0,1), random-init parameters, seeded",
        "config": {"workload": W["name"], "l2": "outputs larger than L2" if W["unit"] == "GB/s"
                   else "inputs and scalograms larger than L2 across a step"},
        "roofline": {"bound": "hbm", "kernel": W["kernels"][dom], "achieved": round(achieved, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "peak_source": peak_src, "algorithmic_bytes_per_call": k_bytes,
                     "call_ms": round(k_ms, 4), "traffic": None,
                     "fwd_ms": round(fwd_ms, 4), "bwd_ms": round(bwd_ms, 4)},
        "gpu_launches": int(launches),
        "e2e": None,
        "clocks": clk.summary(),
    }
    if cpu_line is not None:
        line["cpu_baseline"] = cpu_line
    print(json.dumps(line), flush=True)
    return 0


def run_config_reference(args):
    import torch
    W = WORKLOADS[args.config]()
    torch.set_num_threads(os.cpu_count() or 1)
    times = []
    steps, warmup = args.steps, args.warmup
    for i in range(warmup + steps):
        t = W["cpu"](W["cpu_rows"])
        if i >= warmup:
            times.append(t)
        if t > 5.0:  # a heavy sample: keep the whole run within a few minutes
            steps, warmup = min(steps, 2), min(warmup, i)
            if len(times) >= steps:
                break
    tc = statistics.mean(times) if times else t
    units = W.get("cpu_unit_per_row")
    per = (W["cpu_rows"] * units) if units else W["per_step"] * W["cpu_rows"] / W["rows"]
    value = per / tc / (1e9 if W["unit"] == "GB/s" else 1)
    sample = (f"{W['cpu_rows']} {'batch entries' if units else 'rows'} per step through the fp64 "
              f"CPU oracle port of the reference's CPU path (torch, {os.cpu_count()} threads)")
    return {"metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": W["unit"],
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(tc * 1e3, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic i.i.d. N(0,1)",
            "config": {"workload": W["name"] + " (bounded sample)"},
            "cpu_baseline": {"value": round(value, 4), "unit": W["unit"],
                             "cores": os.cpu_count(), "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 4), "unit": W["unit"], "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}



def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-rows", type=int, default=2048)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--rows", type=int, default=None,
                    help="cfg2, cfg3, cfg3l: rows per GPU (default: the config's; fewer for "
                         "profiling)")
    ap.add_argument("--config", default="cfg2", choices=["cfg2"] + sorted(WORKLOADS),
                    help="cfg2 (default, the headline line) or another baseline config")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.config != "cfg2":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps(run_config_reference(args)), flush=True)
            return 0
        return run_config(args, rank, world, local_rank)

    if args.impl == "reference":
        if rank != 0:
            return 0
        pool = CpuPool(os.cpu_count() or 1)
        try:
            print(json.dumps(run_reference(args, pool)), flush=True)
        finally:
            pool.close()
        return 0

    # CPU pool first (spawned before the first CUDA call), rank 0 at N=1 only
    pool = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        pool = CpuPool(os.cpu_count() or 1)
    import torch
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        line = run_ours(args, rank, world, local_rank, pool)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if pool is not None:
            pool.close()
        if world > 1:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
