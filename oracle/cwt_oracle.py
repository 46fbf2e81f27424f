"""Morlet CWT oracle in torch CPU fp64 (TEST INFRASTRUCTURE ONLY).

Restates the reference's CPU path of the Morlet transform and the three scalogram consumers:

* ``Plan`` -- octave grouping, supports, margins, centre and half-band of ``MorletPlan``
  (``fdwt/cwt.py:88-139``) and the half-band design ``_halfband`` (``fdwt/cwt.py:65-68``);
* ``Plan.filters`` -- the sampled Morlet filters (``fdwt/cwt.py:181-203``);
* ``fb_conv`` -- ``y[r, f, n] = sum_k h[f, k] x[r, n + off - dil k]`` (zero outside the row),
  the filter-bank convolution of ``fdwt/reference.py:52-66``, written as an explicit tap loop;
* ``transform`` -- the octave pyramid of ``fdwt/cwt.py:562-583`` (Morlet stage per octave,
  dilated half-band step between octaves, user scale order restored);
* ``mix`` / ``spectral_softmax`` -- the CPU definitions of ``fdwt/cwt.py:391-394, 545-549``;
* ``token_mixer`` / ``attention`` / ``channel_mix_attention`` -- the layer glue of
  ``fdwt/layers.py:66-72, 155-162, 216-218, 257-262``.

Every function is differentiable with torch autograd, which provides the oracle gradients.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List

import numpy as np
import torch

PI_M14 = math.pi ** -0.25


def freqs_to_scales(freqs, fs: float = 1.0, w0: float = 6.0) -> List[float]:
    f = np.asarray(freqs, dtype=np.float64).reshape(-1)
    return [float(v) for v in w0 * fs / (2 * math.pi * f)]


def halfband(c: int, beta: float) -> torch.Tensor:
    n = torch.arange(-c, c + 1, dtype=torch.float64)
    h = 0.5 * torch.sinc(n / 2) * torch.from_numpy(np.kaiser(2 * c + 1, beta))
    return h / h.sum()


@dataclass
class Stage:
    octave: int
    dil: int
    scale_idx: List[int]
    half: int
    support: List[int]


@dataclass
class Plan:
    scales: List[float]
    w0: float = 6.0
    truncate: float = 4.0
    norm: str = "l2"
    complex: bool = True
    method: str = "fast"
    support_margin: float = 1.0
    stages: List[Stage] = field(default_factory=list)

    def __post_init__(self):
        reach = self.truncate * self.support_margin
        self.channels = 2 if self.complex else 1
        s_th = (self.w0 + self.truncate) / (0.8 * math.pi)
        groups: Dict[int, List[int]] = {}
        for i, s in enumerate(self.scales):
            j = 0 if self.method != "fast" else max(0, math.floor(math.log2(s / s_th)))
            groups.setdefault(j, []).append(i)
        for j in sorted(groups):
            dil = 2 ** j
            sup = {i: max(1, math.ceil(reach * self.scales[i] / dil)) for i in groups[j]}
            order = sorted(groups[j], key=lambda i: sup[i])
            self.stages.append(Stage(j, dil, order, max(sup.values()), [sup[i] for i in order]))
        self.n_octaves = self.stages[-1].octave + 1
        self.center = max(st.half for st in self.stages)
        self.dil = [0.0] * len(self.scales)
        self.sup = [0.0] * len(self.scales)
        for st in self.stages:
            for i, c in zip(st.scale_idx, st.support):
                self.dil[i], self.sup[i] = float(st.dil), float(c)
        c_lp, beta = (16, 8.0) if self.truncate <= 4.5 else (24, 10.0)
        multi = self.n_octaves > 1
        self.lowpass = halfband(c_lp, beta) if multi else torch.zeros(1, dtype=torch.float64)
        self.c_lp = c_lp if multi else 0
        J = self.n_octaves - 1
        by_oct = {st.octave: st for st in self.stages}
        self.margins = [0] * (J + 1)
        for j in range(J, 0, -1):
            own = by_oct[j].half * 2 ** j if j in by_oct else 0
            nxt = self.margins[j + 1] + self.c_lp * 2 ** j if j < J else 0
            self.margins[j] = max(own, nxt)

    @property
    def num_scales(self) -> int:
        return len(self.scales)

    def filters(self, scales: torch.Tensor, w0) -> torch.Tensor:
        """``(S*C, 2*center+1)`` fp64 filters, row ``i*C + c``; differentiable."""
        f64 = torch.float64
        s = scales.to(f64)[:, None]
        dil = torch.tensor(self.dil, dtype=f64)[:, None]
        sup = torch.tensor(self.sup, dtype=f64)[:, None]
        k = torch.arange(-self.center, self.center + 1, dtype=f64)[None, :]
        t = k * dil / s
        env = torch.exp(-0.5 * t * t) * (k.abs() <= sup)
        amp = PI_M14 * dil / (s.sqrt() if self.norm == "l2" else s)
        w0_ = torch.as_tensor(w0, dtype=f64)
        re = (torch.cos(w0_ * t) - torch.exp(-0.5 * w0_ * w0_)) * env * amp
        if not self.complex:
            return re
        im = torch.sin(w0_ * t) * env * amp
        return torch.stack([re, im], 1).reshape(-1, k.shape[1])


def fb_conv(x: torch.Tensor, h: torch.Tensor, n_out: int, off: int, dil: int = 1) -> torch.Tensor:
    """``y[r, f, n] = sum_k h[f, k] x[r, n + off - dil k]``, x zero outside ``[0, N)``."""
    R, N = x.shape
    Fn, K = h.shape
    n = torch.arange(n_out)
    y = x.new_zeros((R, Fn, n_out))
    for k in range(K):
        pos = n + off - dil * k
        valid = (pos >= 0) & (pos < N)
        if not bool(valid.any()):
            continue
        xs = torch.where(valid[None, :], x[:, pos.clamp(0, N - 1)], x.new_zeros(()))
        y = y + h[:, k][None, :, None] * xs[:, None, :]
    return y


def transform(x: torch.Tensor, plan: Plan, H: torch.Tensor) -> torch.Tensor:
    """``x (R, N)`` -> ``(R, S, N, C)`` (C = 2 interleaved re/im, or 1)."""
    R, N = x.shape
    C = plan.channels
    out = [None] * plan.num_scales
    lp = plan.lowpass.to(x.dtype)
    by_oct = {st.octave: st for st in plan.stages}
    xj = x
    for j in range(plan.n_octaves):
        dil, mj = 2 ** j, plan.margins[j]
        if j in by_oct:
            st = by_oct[j]
            rows = [i * C + c for i in st.scale_idx for c in range(C)]
            h = H[rows][:, plan.center - st.half: plan.center + st.half + 1]
            y = fb_conv(xj, h, N, mj + st.half * dil, dil)            # (R, S_j*C, N)
            y = y.reshape(R, len(st.scale_idx), C, N).transpose(-1, -2)
            for k, i in enumerate(st.scale_idx):
                out[i] = y[:, k]
        if j + 1 < plan.n_octaves:
            m1 = plan.margins[j + 1]
            xj = fb_conv(xj, lp[None], N + 2 * m1, mj - m1 + plan.c_lp * dil, dil)[:, 0]
    return torch.stack(out, 1)


def apply_plan(x: torch.Tensor, plan: Plan, H: torch.Tensor) -> torch.Tensor:
    """``(..., N)`` -> ``(..., S, N)`` complex (or real), like ``fdwt/cwt.py:600-612``."""
    lead, N = x.shape[:-1], x.shape[-1]
    y = transform(x.reshape(-1, N).to(torch.float64), plan, H.to(torch.float64))
    y = y.reshape(*lead, plan.num_scales, N, plan.channels)
    return torch.view_as_complex(y.contiguous()) if plan.complex else y[..., 0]


def mix(x: torch.Tensor, plan: Plan, H: torch.Tensor, a: torch.Tensor, b: torch.Tensor):
    """``x (B, D, N)`` -> ``sum_s a[d,s] |W_s| + b[d,s] Re W_s``."""
    w = apply_plan(x, plan, H)
    re = w.real if plan.complex else w
    return torch.einsum("bdsn,ds->bdn", w.abs(), a.to(torch.float64)) + \
        torch.einsum("bdsn,ds->bdn", re, b.to(torch.float64))


def spectral_softmax(x: torch.Tensor, plan: Plan, H: torch.Tensor, V: torch.Tensor, nch: int,
                     tau: float) -> torch.Tensor:
    """``x (R, N)`` -> ``sum_f softmax_f(|W_f x| / tau) V_f`` with V ``(nch, S)`` or ``(G, S, N)``."""
    R, N = x.shape
    p = torch.softmax(apply_plan(x, plan, H).abs() / tau, dim=-2)
    p = p.view(-1, nch, p.shape[1], N)
    V = V.to(torch.float64)
    Vb = V[None, :, :, None] if V.dim() == 2 else V[:, None]
    return (p * Vb).sum(2).reshape(R, N)


def token_mixer(x, plan, H, mag_weight, phase_weight, bias, w_out, b_out):
    """MorletTokenMixer forward on ``x (B, L, D)``."""
    y = mix(x.transpose(1, 2), plan, H, mag_weight, phase_weight).transpose(1, 2) + bias
    return y @ w_out.t() + b_out


def attention(x, plan, H, freq_weight, tau):
    B, Hh, C, T, D = x.shape
    return spectral_softmax(x.reshape(B * Hh * C, T * D), plan, H, freq_weight, C, tau
                            ).reshape(B, Hh, C, T, D)


def channel_mix_attention(x, plan, H, freq_to_channel, tau):
    B, Hh, C, T, D = x.shape
    v = x.reshape(B, Hh, C, T * D).to(torch.float64)
    U = torch.einsum("fk,bhkn->bhfn", freq_to_channel.to(torch.float64), v)
    return spectral_softmax(x.reshape(B * Hh * C, T * D), plan, H,
                            U.reshape(B * Hh, -1, T * D), C, tau).reshape(B, Hh, C, T, D)
