#!/usr/bin/env python
"""Benchmark of the wavelet filter-bank hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config all|cfg1|cfg2|cfg3|cfg3l|cfg4|cfg5|cfg5c]

Headline (configs[1] of the baseline, the one the metric is quoted on): db8 ``periodization``
level-8 ``wavedec`` of x float32 (16, 128, 65536) i.i.d. N(0,1), ``waverec`` of the
coefficients, and the autograd backward through both.  One step = those four multilevel
transforms over the whole batch; arrays of 512 MiB, larger than the 126 MB L2.  ``value`` is the
whole-job algorithmic HBM throughput in GB/s (unique bytes the four transforms must read and
write), device-timed with CUDA events over K steps, max over ranks.  Each rank runs the full
config on its own data ("weak" scaling: rows shard with no collective); at N > 1 the line also
carries ``strong_scaling`` (the config's batch split over the ranks) and ``gather`` (the
optional NCCL all-gather of the per-rank results, timed apart).

The same line carries ``configs``: every other baseline config (cfg1, cfg3, cfg3 learnable,
cfg4, cfg5 and its channel-mix variant), each measured the same way with its own roofline
(HBM bytes, or FP32 FMA work for the fused mixers), ``e2e`` and CPU baseline, and
``mode_sweep``: the headline shape's wavedec and waverec calls in each of the five boundary
modes.

CPU baseline and the reference arm (``--impl reference``): the reference package's own CPU
PyTorch path (``fdwt`` installed under ``baseline/_ref``, called with CPU tensors, all host
threads), on a bounded sample of each workload (rows or batch entries: the ops are row-wise, so
the sample's per-unit cost is the workload's).  Without ``baseline/_ref`` the oracle port in
``oracle/`` stands in and ``kind`` says "port".
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "DWT/CWT achieved HBM GB/s (% of B200 peak); Morlet mixer tokens/s fwd+bwd"
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) per full-size launch of the finest analysis and synthesis passes,
# from one ncu capture of each on 1024 of the 2048 rows scaled by 2 (traffic grows with the
# rows); the captures are summarised in profiles/dwt_cfg2_kernels.txt
TRAFFIC_PER_LAUNCH = {
    "dwt_ana3_stream_kernel<float,16>": 973_150_000,
    "dwt_syn2_stream_kernel<float,16,0>": 970_000_000,
}
CONFIG_NAMES = ["cfg1", "cfg3", "cfg3l", "cfg4", "cfg5", "cfg5c"]


# ------------------------------------------------------------------------------ helpers

def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def fp32_fma_peak(dev):
    """FP32 (non-tensor) peak of this GPU, measured: cuBLAS SGEMM 8192^3 with TF32 off, best
    of 5 (GFLOP/s).  The denominator of the fused mixers' FMA roofline."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        n = 8192
        a = torch.randn(n, n, device=dev)
        b = torch.randn(n, n, device=dev)
        c = a @ b
        best = float("inf")
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b, c
        return 2.0 * n ** 3 / (best / 1e3) / 1e9
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


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


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ------------------------------------------------------------------------------ CPU baselines

_REF = None


def reference_package():
    """The reference package (import name ``fdwt``) installed under ``baseline/_ref``, or None.
    Its CPU path runs when it is given CPU tensors."""
    global _REF
    if _REF is None:
        path = os.path.join(ROOT, "baseline", "_ref")
        _REF = False
        if os.path.isdir(os.path.join(path, "fdwt")):
            sys.path.insert(0, path)
            try:
                _REF = importlib.import_module("fdwt")
            except Exception:
                _REF = False
            finally:
                sys.path.remove(path)
    return _REF or None


def _explicit_bank(name):
    """(dec_lo, dec_hi, rec_lo, rec_hi) lists of a Daubechies bank: PyWavelets (which the
    reference needs for names) is absent, so both packages get the same explicit bank."""
    from pytorch_morlet_fdwt_b200.wavelets import get_filter_bank
    b = get_filter_bank(name)
    return (list(b.dec_lo), list(b.dec_hi), list(b.rec_lo), list(b.rec_hi))


def cpu_time(fn, reps):
    """Median wall time of `reps` calls of fn() after one warm-up call."""
    fn()
    times = []
    for _ in range(reps):
        t = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t)
    return statistics.median(times), times


# ------------------------------------------------------------------------------ workloads
#
# A workload knows its GPU step (forward + backward, split for timing), its dominant kernel
# (timed alone for the roofline), its algorithmic units, and the reference CPU path on a
# bounded sample.  `batch` is the number of batch entries a rank runs (the config's, or its
# share under strong scaling).


def _dwt_lens(n, L, mode, level):
    from pytorch_morlet_fdwt_b200.dwt import dwt_coeff_len
    lens, cur = [], n
    for _ in range(level):
        cur = dwt_coeff_len(cur, L, mode)
        lens.append(cur)
    return lens


def _fma_per_position(plan):
    """Algorithmic FMAs of one forward filter-bank pass per signal position: a complex scale
    with half-support c costs 2c + 1 FMAs after folding the even real and odd imaginary taps
    (one FMA per tap pair for each of re and im, plus the centre)."""
    return sum(2 * c + 1 for st in plan.stages for c in st.support)


class Workload:
    key = ""
    unit = "GB/s"
    batch = 1
    dtype = "f32"

    def units(self, batch):            # algorithmic units of one step on `batch` entries
        raise NotImplementedError

    def setup(self, dev, batch):
        raise NotImplementedError

    def fwd(self, st):
        raise NotImplementedError

    def bwd(self, st):
        pass

    def e2e_step(self, st, x):         # full step on an uploaded input; returns the download
        raise NotImplementedError

    def kernel(self, st):              # (name, callable running the dominant kernel once,
        raise NotImplementedError      #  algorithmic work per call, "hbm" | "fma")

    def cpu(self, ref, sample):        # seconds of the CPU path on `sample` entries
        raise NotImplementedError

    cpu_sample = 1
    cpu_sample_unit = "batch entries"


class Cfg2(Workload):
    key = "cfg2"
    batch = 16
    shape = (128, 65536)
    wavelet, mode, level = "db8", "periodization", 8
    name = ("cfg2: db8 periodization level-8 wavedec + waverec + backward through both, x "
            "float32 (16, 128, 65536)")
    cpu_sample = 64
    cpu_sample_unit = "rows"

    def dir_bytes_per_row(self):
        n = self.shape[-1]
        lens = _dwt_lens(n, 16, self.mode, self.level)
        return (n + sum(lens) + lens[-1]) * 4

    def units(self, batch):
        return 4 * self.dir_bytes_per_row() * batch * self.shape[0]

    def setup(self, dev, batch, rows=None):
        import torch
        import pytorch_morlet_fdwt_b200 as F
        shape = (batch,) + self.shape if rows is None else (1, rows, self.shape[-1])
        st = {"bank": F.get_filter_bank(self.wavelet), "F": F}
        st["x"] = torch.randn(shape, device=dev).requires_grad_()
        st["gy"] = torch.randn(shape, device=dev)
        return st

    def fwd(self, st):
        F = st["F"]
        st["c"] = F.wavedec(st["x"], st["bank"], self.mode, self.level)
        st["y"] = F.waverec(st["c"], st["bank"], self.mode)

    def bwd(self, st):
        import torch
        st["x"].grad = None
        torch.autograd.backward(st["y"], st["gy"])

    def e2e_step(self, st, x):
        import torch
        F = st["F"]
        y = F.waverec(F.wavedec(x, st["bank"], self.mode, self.level), st["bank"], self.mode)
        torch.autograd.backward(y, st["gy"])
        return x.grad

    def kernels(self, st):
        """The finest pass of the step's analysis (levels 1-3 in one launch) and of its
        synthesis (levels 2-1 in one launch)."""
        F = st["F"]
        x2 = st["x"].detach().reshape(-1, self.shape[-1])
        c2 = F.wavedec(x2, st["bank"], self.mode, 2)
        return {"dwt_ana3_stream_kernel<float,16>":
                lambda: F.wavedec(x2, st["bank"], self.mode, 3),
                "dwt_syn2_stream_kernel<float,16,0>":
                lambda: F.waverec(c2, st["bank"], self.mode)}

    def cpu(self, ref, sample):
        import torch
        if ref is None:
            from oracle import dwt_oracle as D
            tb = _explicit_bank(self.wavelet)
            x = np.random.default_rng(0).standard_normal((sample, self.shape[-1])).astype(
                np.float32)
            t = time.perf_counter()
            c = D.wavedec(x, tb, self.mode, self.level)
            y = D.waverec(c, tb, self.mode)
            gc = D.waverec_vjp(c, y, tb, self.mode)
            D.wavedec_vjp(x.shape[-1], gc, tb, self.mode)
            return time.perf_counter() - t
        bank = _explicit_bank(self.wavelet)
        x = torch.randn(sample, self.shape[-1], requires_grad=True)
        gy = torch.randn(sample, self.shape[-1])
        t = time.perf_counter()
        y = ref.waverec(ref.wavedec(x, bank, self.mode, self.level), bank, self.mode)
        torch.autograd.backward(y, gy)
        return time.perf_counter() - t

    def cpu_units(self, sample):
        return 4 * self.dir_bytes_per_row() * sample


class Cfg1(Workload):
    key = "cfg1"
    graph = True  # launch-bound: also timed as a CUDA-graph replay
    batch = 32
    shape = (64, 2500)
    name = ("cfg1: db4 symmetric level-5 wavedec, its backward of sum(coeffs^2), and waverec, "
            "x float32 (32, 64, 2500)")
    cpu_sample = 32

    def dir_bytes_per_row(self):
        n = self.shape[-1]
        lens = _dwt_lens(n, 8, "symmetric", 5)
        return (n + sum(lens) + lens[-1]) * 4

    def units(self, batch):
        return 3 * self.dir_bytes_per_row() * batch * self.shape[0]

    def setup(self, dev, batch):
        import torch
        import pytorch_morlet_fdwt_b200 as F
        return {"F": F, "bank": F.get_filter_bank("db4"),
                "x": torch.randn((batch,) + self.shape, device=dev).requires_grad_()}

    def fwd(self, st):
        F = st["F"]
        st["c"] = F.wavedec(st["x"], st["bank"], "symmetric", 5)
        st["y"] = F.waverec([c.detach() for c in st["c"]], st["bank"], "symmetric")

    def bwd(self, st):
        st["x"].grad = None
        sum(c.square().sum() for c in st["c"]).backward()

    def e2e_step(self, st, x):
        F = st["F"]
        c = F.wavedec(x, st["bank"], "symmetric", 5)
        st["y"] = F.waverec([v.detach() for v in c], st["bank"], "symmetric")
        sum(v.square().sum() for v in c).backward()
        return x.grad

    def kernel(self, st):
        F = st["F"]
        return ("wavedec call: dwt_analysis_kernel<float> (all five levels in one launch)",
                lambda: F.wavedec(st["x"].detach(), st["bank"], "symmetric", 5),
                self.dir_bytes_per_row() * st["x"].shape[0] * self.shape[0], "hbm")

    def cpu(self, ref, sample):
        import torch
        bank = _explicit_bank("db4")
        mod = ref if ref is not None else None
        x = torch.randn((sample,) + self.shape, requires_grad=True)
        if mod is None:
            from oracle import dwt_oracle as D
            xn = x.detach().reshape(-1, self.shape[-1]).numpy()
            t = time.perf_counter()
            c = D.wavedec(xn, bank, "symmetric", 5)
            D.waverec(c, bank, "symmetric")
            D.wavedec_vjp(self.shape[-1], [2 * v for v in c], bank, "symmetric")
            return time.perf_counter() - t
        t = time.perf_counter()
        c = mod.wavedec(x, bank, "symmetric", 5)
        mod.waverec([v.detach() for v in c], bank, "symmetric")
        sum(v.square().sum() for v in c).backward()
        return time.perf_counter() - t

    def cpu_units(self, sample):
        return self.units(sample)


class Cfg3(Workload):
    batch = 32
    shape = (64, 2500)

    def __init__(self, learnable):
        self.learnable = learnable
        self.key = "cfg3l" if learnable else "cfg3"
        self.name = ("cfg3: Morlet CWT fast, 40 freqs logspace(-0.3,2) @ 250 Hz, l1, x float32 "
                     "(32, 64, 2500) -> complex64 (32, 64, 40, 2500)")
        if learnable:
            self.name += "; learnable scales and w0, forward + backward of sum |W|^2"
        self.cpu_sample = 1 if learnable else 4

    def _bytes(self, batch):
        rows = batch * self.shape[0]
        x = rows * self.shape[1] * 4
        w = rows * 40 * self.shape[1] * 8
        return x, w

    def units(self, batch):
        x, w = self._bytes(batch)
        return x + w + (w + 2 * x if self.learnable else 0)

    def _module(self, F):
        return F.CWT1D(freqs=np.logspace(-0.3, 2, 40), fs=250.0, norm="l1",
                       learnable=self.learnable, learnable_w0=self.learnable)

    def setup(self, dev, batch):
        import torch
        import pytorch_morlet_fdwt_b200 as F
        torch.manual_seed(0)
        m = self._module(F).to(dev)
        return {"m": m, "x": torch.randn((batch,) + self.shape,
                                         device=dev).requires_grad_(self.learnable)}

    def fwd(self, st):
        st["y"] = st["m"](st["x"])

    def bwd(self, st):
        import torch
        if self.learnable:
            st["x"].grad = None
            st["m"].zero_grad()
            torch.view_as_real(st["y"]).square().sum().backward()

    def e2e_step(self, st, x):
        import torch
        if not self.learnable:
            return torch.view_as_real(st["m"](x.detach()))
        st["m"].zero_grad()
        torch.view_as_real(st["m"](x)).square().sum().backward()
        return x.grad

    def kernel(self, st):
        import torch
        from pytorch_morlet_fdwt_b200.cwt import _cwt_backward, _cwt_forward
        m = st["m"]
        x2 = st["x"].detach().reshape(-1, self.shape[1])
        H = m._filters(x2.device, torch.float32).detach()
        xb, wb = self._bytes(st["x"].shape[0])
        if not self.learnable:
            return ("cwt_forward_kernel<float,float,0>", lambda: _cwt_forward(x2, m.plan, H),
                    xb + wb, "hbm")
        g = torch.randn((x2.shape[0], 40, self.shape[1], 2), device=x2.device)
        return ("cwt_backward_kernel<float,0> + reduce_rows_kernel (dL/dx and dL/dH)",
                lambda: _cwt_backward(g, x2, m.plan, H, True, True), wb + 2 * xb, "hbm")

    def cpu(self, ref, sample):
        import torch
        x = torch.randn((sample,) + self.shape, requires_grad=self.learnable)
        if ref is None:
            import pytorch_morlet_fdwt_b200 as F
            from oracle import cwt_oracle as C
            m = self._module(F)
            po = C.Plan(m.plan.scales, norm="l1", support_margin=1.25 if self.learnable else 1.0)
            ls = m.log_scales.detach().double().requires_grad_(self.learnable)
            w0 = torch.tensor(6.0, dtype=torch.float64, requires_grad=self.learnable)
            t = time.perf_counter()
            W = C.apply_plan(x.detach().double().requires_grad_(self.learnable), po,
                             po.filters(ls.exp(), w0))
            if self.learnable:
                W.abs().square().sum().backward()
            return time.perf_counter() - t
        m = self._module(ref)
        t = time.perf_counter()
        W = m(x)
        if self.learnable:
            torch.view_as_real(W).square().sum().backward()
        return time.perf_counter() - t

    def cpu_units(self, sample):
        return self.units(sample)


class Cfg4(Workload):
    key = "cfg4"
    unit = "tokens/s"
    batch = 8
    shape = (4096, 256)
    name = ("cfg4: MorletTokenMixer dim 256, 16 freqs logspace(0,1.8) @ 250 Hz, x float32 "
            "(8, 4096, 256), forward + backward of sum(y^2)")

    def units(self, batch):
        return batch * self.shape[0]

    def _module(self, F):
        import torch
        torch.manual_seed(0)
        return F.MorletTokenMixer(256, freqs=np.logspace(0, 1.8, 16).tolist(), fs=250)

    def setup(self, dev, batch):
        import torch
        import pytorch_morlet_fdwt_b200 as F
        m = self._module(F).to(dev)
        return {"m": m, "x": torch.randn((batch,) + self.shape, device=dev).requires_grad_()}

    def fwd(self, st):
        st["y"] = st["m"](st["x"])

    def bwd(self, st):
        st["x"].grad = None
        st["m"].zero_grad()
        st["y"].square().sum().backward()

    def e2e_step(self, st, x):
        st["m"].zero_grad()
        st["m"](x).square().sum().backward()
        return x.grad

    def kernel(self, st):
        import torch
        from pytorch_morlet_fdwt_b200.cwt import _mix_tokens_backward
        m = st["m"]
        x = st["x"].detach()  # (B, L, D) tokens, read in place by the kernels
        H = m.cwt._filters(x.device, torch.float32).detach()
        gy = torch.randn_like(x)
        a, b = m.mag_weight.detach(), m.phase_weight.detach()
        fma = 4 * _fma_per_position(m.cwt.plan) * x.numel()
        return ("cwt_backward_kernel<float,1> + tokens_to_rows_kernel + reduce_rows_kernel (mix "
                "backward on the token layout: recompute, adjoint, filter gradient)",
                lambda: _mix_tokens_backward(gy, x, m.cwt.plan, H, a, b, True, True, True), fma,
                "fma")

    def cpu(self, ref, sample):
        import torch
        x = torch.randn((sample,) + self.shape, requires_grad=True)
        if ref is None:
            import pytorch_morlet_fdwt_b200 as F
            from oracle import cwt_oracle as C
            m = self._module(F).double()
            po = C.Plan(m.cwt.plan.scales, support_margin=1.25)
            ls = m.cwt.log_scales.detach().double().requires_grad_()
            xd = x.detach().double().requires_grad_()
            t = time.perf_counter()
            y = C.token_mixer(xd, po, po.filters(ls.exp(), m.cwt.w0_value), m.mag_weight,
                              m.phase_weight, m.bias, m.out_proj.weight, m.out_proj.bias)
            y.square().sum().backward()
            return time.perf_counter() - t
        m = self._module(ref)
        t = time.perf_counter()
        m(x).square().sum().backward()
        return time.perf_counter() - t

    def cpu_units(self, sample):
        return self.units(sample)


class Cfg5(Workload):
    unit = "tokens/s"
    batch = 64
    shape = (4, 19, 30, 200)

    def __init__(self, channel_mix):
        self.channel_mix = channel_mix
        self.key = "cfg5c" if channel_mix else "cfg5"
        self.name = ("cfg5: Morlet" + ("ChannelMix" if channel_mix else "") + "Attention, 19 "
                     "channels, hidden 200, x float32 (64, 4, 19, 30, 200), forward + backward "
                     "of sum(y^2)")

    def units(self, batch):  # tokens = B * C * T patches
        return batch * 19 * 30

    def _module(self, F):
        import torch
        torch.manual_seed(0)
        cls = F.MorletChannelMixAttention if self.channel_mix else F.MorletAttention
        return cls(num_channels=19, hidden_dim=200)

    def setup(self, dev, batch):
        import torch
        import pytorch_morlet_fdwt_b200 as F
        m = self._module(F).to(dev)
        return {"m": m, "x": torch.randn((batch,) + self.shape, device=dev).requires_grad_()}

    fwd = Cfg4.fwd
    bwd = Cfg4.bwd
    e2e_step = Cfg4.e2e_step

    def kernel(self, st):
        import torch
        from pytorch_morlet_fdwt_b200.cwt import _softmax_backward, _softmax_forward
        m = st["m"]
        x = st["x"].detach()
        B = x.shape[0]
        x2 = x.reshape(-1, 6000)
        H = m.cwt._filters(x2.device, torch.float32).detach()
        if self.channel_mix:
            v = x.reshape(B, 4, 19, 6000)
            V = torch.einsum("fk,bhkn->bhfn", m.freq_to_channel.detach(), v).reshape(B * 4, 16,
                                                                                      6000)
        else:
            V = m.freq_weight.detach()
        out, mm, ll = _softmax_forward(x2, m.cwt.plan, H, V, 19, m.temperature)
        g = torch.randn_like(out)
        fma = 4 * _fma_per_position(m.cwt.plan) * x2.numel()
        return ("cwt_backward_kernel<float,2> + reduce_rows_kernel (spectral softmax backward: "
                "recompute, adjoint, filter gradient)",
                lambda: _softmax_backward(g, x2, m.cwt.plan, H, V, 19, m.temperature, mm, ll, out,
                                          True, True), fma, "fma")

    def cpu(self, ref, sample):
        import torch
        x = torch.randn((sample,) + self.shape, requires_grad=True)
        if ref is None:
            import pytorch_morlet_fdwt_b200 as F
            from oracle import cwt_oracle as C
            m = self._module(F).double()
            po = C.Plan(m.cwt.plan.scales, support_margin=1.25)
            ls = m.cwt.log_scales.detach().double().requires_grad_()
            w0 = torch.tensor(m.cwt.w0_value, dtype=torch.float64, requires_grad=True)
            xd = x.detach().double().requires_grad_()
            t = time.perf_counter()
            H = po.filters(ls.exp(), w0)
            if self.channel_mix:
                y = C.channel_mix_attention(xd, po, H, m.freq_to_channel, m.temperature)
            else:
                y = C.attention(xd, po, H, m.freq_weight, m.temperature)
            y.square().sum().backward()
            return time.perf_counter() - t
        m = self._module(ref)
        t = time.perf_counter()
        m(x).square().sum().backward()
        return time.perf_counter() - t

    def cpu_units(self, sample):
        return self.units(sample)


WORKLOADS = {"cfg1": Cfg1(), "cfg2": Cfg2(), "cfg3": Cfg3(False), "cfg3l": Cfg3(True),
             "cfg4": Cfg4(), "cfg5": Cfg5(False), "cfg5c": Cfg5(True)}


def cpu_baseline(W, reps=3):
    """The reference's CPU path (or the port) on the workload's bounded sample, all host
    threads; returns the cpu_baseline object."""
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ref = reference_package()
    kind = "reference" if ref is not None else "port"
    sample = W.cpu_sample
    t, _ = cpu_time(lambda: W.cpu(ref, sample), reps)
    units = W.cpu_units(sample)
    scale = 1e9 if W.unit == "GB/s" else 1.0
    what = ("the reference package's CPU PyTorch path (fdwt from baseline/_ref, CPU tensors)"
            if ref is not None else "the fp64 CPU oracle port of the reference's CPU path")
    return {"value": round(units / t / scale, 4), "unit": W.unit, "cores": threads,
            "kind": kind, "cpu": cpu_model(),
            "sample": f"{sample} {W.cpu_sample_unit} of the workload per step through {what}, "
                      f"{threads} threads, median of {reps} after 1 warm-up ({t:.3f} s each)"}


# ------------------------------------------------------------------------------ GPU timing

def time_steps(W, st, steps, warmup, world, dev, barrier):
    """Device time (ms) of `steps` fwd+bwd steps, and the mean fwd / bwd call times; max over
    ranks.  Also the launches of this library inside the timed region."""
    import torch
    from pytorch_morlet_fdwt_b200 import _lib
    for _ in range(warmup):  # the timed loop's own body (see run_headline)
        W.fwd(st)
        W.bwd(st)
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    barrier()
    torch.cuda.synchronize()
    l0 = _lib.launch_count()
    for e in ev:
        e[0].record()
        W.fwd(st)
        e[1].record()
        W.bwd(st)
        e[2].record()
    torch.cuda.synchronize()
    launches = _lib.launch_count() - l0
    barrier()
    ms = ev[0][0].elapsed_time(ev[-1][2])
    fwd = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    bwd = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    ms, fwd, bwd = max_over_ranks([ms, fwd, bwd], world, dev)
    return ms, fwd, bwd, launches


def time_graph(W, st, steps, world, dev, barrier):
    """The fwd+bwd step captured once in a CUDA graph (torch.cuda.graph) and replayed `steps`
    times: device ms (max over ranks) and this library's launches per replayed step (counted
    while capturing).  For launch-bound shapes, where the eager step measures the host."""
    import torch
    from pytorch_morlet_fdwt_b200 import _lib
    for k in ("c", "y"):  # drop the eager steps' autograd graphs (their AccumulateGrad nodes)
        st.pop(k, None)
    st["x"].grad = None
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            W.fwd(st)
            W.bwd(st)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    l0 = _lib.launch_count()
    with torch.cuda.graph(g):
        W.fwd(st)
        W.bwd(st)
    per_step = _lib.launch_count() - l0
    g.replay()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    (ms,) = max_over_ranks([e0.elapsed_time(e1)], world, dev)
    del g
    return ms, per_step


def time_call(fn, reps, barrier):
    """Mean device time (ms) of one call of fn over `reps` back-to-back calls, and the number of
    this library's launches per call."""
    import torch
    from pytorch_morlet_fdwt_b200 import _lib
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
    return e0.elapsed_time(e1) / reps, (_lib.launch_count() - l0) / reps


def e2e_pipelined(step, x0, steps, warmup, barrier):
    """Device time of `steps` end-to-end steps: every step copies its input from pinned host
    memory (host->device), runs the step through the public API and copies the step's result
    (`step` returns it) back to pinned host memory.  The copies run on their own streams,
    double-buffered, so that step i+1's upload and step i's download overlap step i's kernels
    and each other (PCIe is full duplex); the timed region runs from the first upload to the
    last download.  Returns (ms, d2h bytes per step)."""
    import torch
    dev = x0.device
    xh = x0.detach().cpu().pin_memory()
    xd = [torch.empty_like(x0, requires_grad=False) for _ in range(2)]
    with torch.no_grad():
        xd[0].copy_(x0)
    probe = step(xd[0].detach().requires_grad_(x0.requires_grad))
    gh = [torch.empty(probe.shape, dtype=probe.dtype).pin_memory() for _ in range(2)]
    d2h = probe.numel() * probe.element_size()
    del probe
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event(enable_timing=False)  # noqa: E731

    def run(n, timed):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        uploaded = [ev() for _ in range(n)]
        consumed = [None, None]   # compute done with xd[b]
        computed = [ev() for _ in range(n)]
        downloaded = [None, None]  # gh[b] and the result of the step that used b are free
        results = [None, None]
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
            xe = xd[b].detach().requires_grad_(x0.requires_grad)
            results[b] = step(xe)
            consumed[b] = ev()
            consumed[b].record(comp)
            computed[i].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(computed[i])
                gh[b].copy_(results[b], non_blocking=True)
                downloaded[b] = ev()
                downloaded[b].record(s_out)
        if timed:
            end.record(s_out)
        torch.cuda.synchronize()
        return start.elapsed_time(end) if timed else 0.0

    run(warmup, False)
    barrier()
    torch.cuda.synchronize()
    return run(steps, True), d2h


# ------------------------------------------------------------------------------ our arm

def measure_config(W, args, world, dev, barrier, cpu, fp32_peak, batch=None, full=True):
    """One config's object: value, timing, roofline, e2e (and the given cpu baseline)."""
    import torch
    batch = W.batch if batch is None else batch
    torch.manual_seed(100 + (dev.index or 0))
    st = W.setup(dev, batch)
    steps = args.steps
    ms, fwd, bwd, launches = time_steps(W, st, steps, max(3, args.warmup), world, dev, barrier)
    units = W.units(batch)
    scale = 1e9 if W.unit == "GB/s" else 1.0
    out = {"workload": W.name + ("" if batch == W.batch else f" [batch {batch} per GPU]"),
           "value": round(job_throughput(units, steps, world, ms, scale), 3), "unit": W.unit,
           "ms_per_step": round(ms / steps, 4), "fwd_ms": round(fwd, 4),
           "bwd_ms": round(bwd, 4), "gpu_launches": int(launches),
           "units_per_step_per_gpu": units}
    if getattr(W, "graph", False):
        try:
            g_ms, g_launches = time_graph(W, st, steps, world, dev, barrier)
        except RuntimeError as e:  # capture refused: report it, keep the eager numbers
            g_ms, g_launches = None, repr(e)[:200]
    if getattr(W, "graph", False) and g_ms is None:
        out["graph_replay"] = {"unavailable": g_launches}
    elif getattr(W, "graph", False):
        out["graph_replay"] = {
            "what": "the same fwd+bwd step captured once with torch.cuda.graph and replayed "
                    f"{steps} times (the eager step above is bound by host-side launch "
                    "overhead at this size)",
            "value": round(job_throughput(units, steps, world, g_ms, scale), 3),
            "unit": W.unit, "ms_per_step": round(g_ms / steps, 4),
            "gpu_launches_per_step": int(g_launches)}
    if not full:
        return out
    name, fn, work, bound = W.kernel(st)
    k_ms, per_call = time_call(fn, max(3, steps), barrier)
    (k_ms,) = max_over_ranks([k_ms], world, dev)
    if bound == "hbm":
        peak, src = peaks()
        achieved = work / (k_ms / 1e3) / 1e9
        out["roofline"] = {"bound": "hbm", "kernel": name, "achieved": round(achieved, 1),
                           "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                           "peak_source": src, "algorithmic_bytes_per_call": work,
                           "call_ms": round(k_ms, 4), "launches_per_call": per_call,
                           "traffic": None}
    else:
        achieved = 2 * work / (k_ms / 1e3) / 1e12
        out["roofline"] = {"bound": "fp32 fma", "kernel": name, "achieved": round(achieved, 2),
                           "peak": round(fp32_peak / 1e3, 2), "unit": "TFLOP/s",
                           "frac": round(achieved * 1e3 / fp32_peak, 4),
                           "peak_source": "measured in this run: cuBLAS SGEMM 8192^3, TF32 off",
                           "algorithmic_fma_per_call": work,
                           "fma_count": "4 forward filter-bank passes' worth per position: "
                                        "recompute W and the adjoint (each sum over scales of "
                                        "2 * half-support + 1 FMAs after folding the even/odd "
                                        "taps) and the filter gradient (twice that: separate "
                                        "re and im gradients for every tap, no folding)",
                           "call_ms": round(k_ms, 4), "launches_per_call": per_call,
                           "traffic": None}
    if not args.no_e2e:
        n_e2e = max(2, min(steps, 5))
        e_ms, d2h = e2e_pipelined(lambda x: W.e2e_step(st, x), st["x"], n_e2e, 2, barrier)
        (e_ms,) = max_over_ranks([e_ms], world, dev)
        x = st["x"]
        out["e2e"] = {"value": round(job_throughput(units, n_e2e, world, e_ms, scale), 3),
                      "unit": W.unit, "h2d_bytes_per_step": x.numel() * x.element_size(),
                      "d2h_bytes_per_step": d2h, "ms_per_step": round(e_ms / n_e2e, 3)}
    if cpu is not None:
        out["cpu_baseline"] = cpu
    del st
    torch.cuda.empty_cache()
    return out


def run_headline(args, rank, world, local_rank, cpu):
    import torch
    import torch.distributed as dist
    from pytorch_morlet_fdwt_b200 import _lib
    dev = torch.device("cuda", local_rank)
    W = WORKLOADS["cfg2"]

    def barrier():
        if world > 1:
            dist.barrier()

    torch.manual_seed(1234 + rank)
    st = W.setup(dev, W.batch, rows=args.rows)
    R = st["x"].numel() // W.shape[-1]
    step_bytes = 4 * W.dir_bytes_per_row() * R
    F, bank = st["F"], st["bank"]
    # warm-up runs the timed loop's own body, so that the allocator already holds every block
    # the timed steps reuse (results kept alive elsewhere would make them allocate anew)
    for _ in range(args.warmup):
        st["x"].grad = None
        coeffs = F.wavedec(st["x"], bank, W.mode, W.level)
        y = F.waverec(coeffs, bank, W.mode)
        torch.autograd.backward(y, st["gy"])
    torch.cuda.synchronize()
    ka, kb, kc = ([torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
                  for _ in range(3))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    with ClockSampler(local_rank) as clk:
        start.record()
        for i in range(args.steps):
            st["x"].grad = None
            ka[i].record()
            coeffs = F.wavedec(st["x"], bank, W.mode, W.level)
            kb[i].record()
            y = F.waverec(coeffs, bank, W.mode)
            kc[i].record()
            torch.autograd.backward(y, st["gy"])
        end.record()
        torch.cuda.synchronize()
    launches = _lib.launch_count() - launches0
    barrier()
    ms = start.elapsed_time(end)
    ana_ms = statistics.mean(a.elapsed_time(b) for a, b in zip(ka, kb))
    syn_ms = statistics.mean(b.elapsed_time(c) for b, c in zip(kb, kc))
    ms, ana_ms, syn_ms = max_over_ranks([ms, ana_ms, syn_ms], world, dev)
    kern = {}
    for name, fn in W.kernels(st).items():
        k_ms, per_call = time_call(fn, max(3, args.steps), barrier)
        if per_call != 1:
            raise RuntimeError(f"{name}: a two-level call was not exactly one launch")
        kern[name] = k_ms
    vals = max_over_ranks(list(kern.values()), world, dev)
    kern = dict(zip(kern, vals))
    e2e = None
    if not args.no_e2e:
        n_e2e = max(1, min(args.steps, 10))
        e_ms, d2h = e2e_pipelined(lambda x: W.e2e_step(st, x), st["x"], n_e2e,
                                  max(1, args.warmup // 2), barrier)
        (e_ms,) = max_over_ranks([e_ms], world, dev)
        e2e = {"value": round(step_bytes * n_e2e * world / (e_ms / 1e3) / 1e9, 2),
               "unit": "GB/s", "h2d_bytes_per_step": st["x"].numel() * 4,
               "d2h_bytes_per_step": d2h, "ms_per_step": round(e_ms / n_e2e, 3),
               "copies": "input upload and gradient download of every step on their own "
                         "streams, double-buffered: step i+1's upload and step i's download "
                         "overlap step i's kernels"}
    x_shape = tuple(st["x"].shape)
    del st
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    peak, peak_src = peaks()
    dominant = max(kern, key=kern.get)
    kern_ms = kern[dominant]
    achieved = W.dir_bytes_per_row() * R / (kern_ms / 1e3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(job_throughput(step_bytes, args.steps, world, ms, 1e9), 2),
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
            "workload": W.name + f" per GPU",
            "shape_per_gpu": x_shape,
            "algorithmic_bytes_per_step": step_bytes,
            "l2": "inputs larger than L2 (512 MiB per array)",
            "parallelism": f"rows sharded by rank, {world} GPU(s), no collective",
        },
        "roofline": {
            "bound": "hbm", "kernel": dominant,
            "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": peak_src,
            "algorithmic_bytes_per_launch": W.dir_bytes_per_row() * R,
            "launch_ms": round(kern_ms, 4),
            "traffic": TRAFFIC_PER_LAUNCH.get(dominant),
            "kernels_ms_per_launch": {k: round(v, 4) for k, v in kern.items()},
            "launch": "the finest pass of the step's analysis (levels 1-3) / synthesis "
                      "(levels 2-1), one launch over every row: x (or the level-1 details and "
                      "level-2 coefficients) read once, the other side written once",
            "calls_ms": {"wavedec (8 levels)": round(ana_ms, 4),
                         "waverec (8 levels)": round(syn_ms, 4)},
        },
        "gpu_launches": int(launches),
        "e2e": e2e,
        "clocks": clk.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


def run_mode_sweep(args, world, dev, barrier):
    """The headline shape in each of the five boundary modes: one wavedec and one waverec call
    per mode (forward only: the backward of each call runs the other's kernels), device-timed
    over back-to-back calls, max over ranks.  Bytes per call are the algorithmic ones of that
    mode (x once, every coefficient array once)."""
    import torch
    import pytorch_morlet_fdwt_b200 as F
    W = WORKLOADS["cfg2"]
    bank = F.get_filter_bank(W.wavelet)
    torch.manual_seed(4321 + (dev.index or 0))
    x = torch.randn((W.batch,) + W.shape, device=dev)
    rows = x.numel() // W.shape[-1]
    peak, _ = peaks()
    reps = max(3, args.steps)
    out = {}
    with torch.no_grad():
        for mode in ("periodization", "zero", "periodic", "symmetric", "reflect"):
            lens = _dwt_lens(W.shape[-1], 16, mode, W.level)
            nbytes = (W.shape[-1] + sum(lens) + lens[-1]) * 4 * rows
            c = F.wavedec(x, bank, mode, W.level)
            a_ms, a_l = time_call(lambda: F.wavedec(x, bank, mode, W.level), reps, barrier)
            s_ms, s_l = time_call(lambda: F.waverec(c, bank, mode), reps, barrier)
            a_ms, s_ms = max_over_ranks([a_ms, s_ms], world, dev)
            a_gbs = nbytes * world / (a_ms / 1e3) / 1e9
            s_gbs = nbytes * world / (s_ms / 1e3) / 1e9
            out[mode] = {"bytes_per_call_per_gpu": nbytes,
                         "wavedec_ms": round(a_ms, 4), "wavedec_gbs": round(a_gbs, 1),
                         "wavedec_frac": round(a_gbs / world / peak, 4),
                         "wavedec_launches": a_l,
                         "waverec_ms": round(s_ms, 4), "waverec_gbs": round(s_gbs, 1),
                         "waverec_frac": round(s_gbs / world / peak, 4),
                         "waverec_launches": s_l}
            del c
    del x
    torch.cuda.empty_cache()
    return {"what": "db8 level-8 wavedec / waverec of x float32 (16, 128, 65536) per GPU in "
                    "every boundary mode; GB/s over all GPUs, frac of the measured HBM copy "
                    "bandwidth per GPU", "modes": out}


def run_strong_and_gather(args, rank, world, local_rank):
    """At N > 1: the headline config with its batch split over the ranks (strong scaling), and
    the optional NCCL all-gather of the per-rank input gradients, timed apart."""
    import torch
    import torch.distributed as dist
    from pytorch_morlet_fdwt_b200.sharding import gather_batch, shard_bounds
    dev = torch.device("cuda", local_rank)
    W = WORKLOADS["cfg2"]
    b0, b1 = shard_bounds(W.batch, rank, world)
    res = {}
    if b1 - b0 >= 1 and W.batch % world == 0:
        m = measure_config(W, args, world, dev, dist.barrier, None, None, batch=b1 - b0,
                           full=False)
        m["scaling"] = "strong"
        m["split"] = f"batch {W.batch} over {world} GPUs: {b1 - b0} per GPU"
        res["strong_scaling"] = m
        torch.manual_seed(7 + rank)
        st = W.setup(dev, b1 - b0)
        W.fwd(st)
        W.bwd(st)
        g = st["x"].grad
        for _ in range(2):
            gather_batch(g)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        reps = 5
        for _ in range(reps):
            out = gather_batch(g)
        e1.record()
        torch.cuda.synchronize()
        (g_ms,) = max_over_ranks([e0.elapsed_time(e1) / reps], world, dev)
        nbytes = out.numel() * out.element_size()
        res["gather"] = {"what": "all_gather_into_tensor of every rank's dL/dx shard (NCCL), "
                                 "outside the device-timed step",
                         "bytes": nbytes, "ms": round(g_ms, 4),
                         "algbw_gbs": round(nbytes / (g_ms / 1e3) / 1e9, 1)}
        del st, out
        torch.cuda.empty_cache()
    return res


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    names = CONFIG_NAMES if args.config == "all" else (
        [] if args.config == "cfg2" else [args.config])
    headline = args.config in ("all", "cfg2")
    # the CPU baselines (rank 0 at N=1) run after every GPU measurement: their host threads
    # must not compete with the thread that launches the timed steps
    cpu = {}
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    barrier = dist.barrier if world > 1 else (lambda: None)
    try:
        line = run_headline(args, rank, world, local_rank, None) if headline else None
        if headline and args.rows is None and not args.no_modes:
            sweep = run_mode_sweep(args, world, dev, barrier)
            if line is not None:
                line["mode_sweep"] = sweep
        if world > 1 and headline and args.rows is None:
            extra = run_strong_and_gather(args, rank, world, local_rank)
            if line is not None:
                line.update(extra)
        fp32_peak = fp32_fma_peak(dev) if names else None
        configs = {}
        for k in names:
            configs[k] = measure_config(WORKLOADS[k], args, world, dev, barrier, None, fp32_peak,
                                        batch=args.batch)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            torch.cuda.synchronize()
            if line is not None:
                line["cpu_baseline"] = cpu_baseline(WORKLOADS["cfg2"])
            for k in names:
                configs[k]["cpu_baseline"] = cpu_baseline(WORKLOADS[k])
        if rank == 0:
            if line is None:  # a single non-headline config: its object is the line
                k = names[0]
                c = configs[k]
                line = {"metric": METRIC, "value": c["value"], "unit": c["unit"],
                        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                        "ms_per_step": c["ms_per_step"], "higher_is_better": True,
                        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                        "data": "synthetic i.i.d. N(0,1), random-init parameters, seeded",
                        "config": {"workload": c["workload"]},
                        "roofline": c.get("roofline"), "gpu_launches": c["gpu_launches"],
                        "e2e": c.get("e2e")}
                if "cpu_baseline" in c:
                    line["cpu_baseline"] = c["cpu_baseline"]
                if "graph_replay" in c:
                    line["graph_replay"] = c["graph_replay"]
            elif configs:
                line["configs"] = configs
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------------------ reference arm

def run_reference(args, rank, world):
    """The reference's own CPU path, rank 0 only: the headline config's bounded sample per step
    (all host threads), plus each other config's sample (1 warm-up + 2 steps) when --config
    all."""
    if rank != 0:
        return 0
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ref = reference_package()
    kind = "reference" if ref is not None else "port"
    key = "cfg2" if args.config in ("all", "cfg2") else args.config
    W = WORKLOADS[key]
    times = []
    for i in range(args.warmup + args.steps):
        t = W.cpu(ref, W.cpu_sample)
        if i >= args.warmup:
            times.append(t)
    t = statistics.mean(times)
    scale = 1e9 if W.unit == "GB/s" else 1.0
    value = W.cpu_units(W.cpu_sample) / t / scale
    what = ("the reference package's CPU PyTorch path (fdwt from baseline/_ref, CPU tensors)"
            if ref is not None else "the fp64 CPU oracle port of the reference's CPU path")
    line = {
        "metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": W.unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic i.i.d. N(0,1), seeded",
        "config": {"workload": W.name + (" per GPU" if key == "cfg2" else "")},
        "cpu_baseline": {"value": round(value, 4), "unit": W.unit, "cores": threads,
                         "kind": kind, "cpu": cpu_model(),
                         "sample": f"{W.cpu_sample} {W.cpu_sample_unit} of the workload per "
                                   f"step through {what}, {threads} threads"},
        "e2e": {"value": round(value, 4), "unit": W.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if args.config == "all":
        line["configs"] = {}
        for k in CONFIG_NAMES:
            Wk = WORKLOADS[k]
            tk, _ = cpu_time(lambda: Wk.cpu(ref, Wk.cpu_sample), 2)
            sk = 1e9 if Wk.unit == "GB/s" else 1.0
            line["configs"][k] = {
                "workload": Wk.name, "value": round(Wk.cpu_units(Wk.cpu_sample) / tk / sk, 4),
                "unit": Wk.unit, "kind": kind,
                "sample": f"{Wk.cpu_sample} {Wk.cpu_sample_unit} per step, median of 2 after 1 "
                          f"warm-up ({tk:.3f} s each)"}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="all", choices=["all", "cfg2"] + CONFIG_NAMES,
                    help="all (default: the cfg2 headline line with every other config under "
                         "'configs'), or one config alone")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-modes", action="store_true",
                    help="skip the five-mode sweep of the headline shape")
    ap.add_argument("--rows", type=int, default=None,
                    help="cfg2 only: rows per GPU (default: the config's; fewer for profiling)")
    ap.add_argument("--batch", type=int, default=None,
                    help="the other configs: batch per GPU (default: the config's; smaller for "
                         "profiling)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
