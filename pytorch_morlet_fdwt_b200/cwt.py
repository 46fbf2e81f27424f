"""Continuous wavelet transform with the (complex) Morlet wavelet, on sm_100a kernels.

    W[s, n] = sum_m x[m] * conj(psi((m - n) / s)) / norm(s)
    psi(t)  = pi^(-1/4) * (exp(i*w0*t) - exp(-w0^2/2)) * exp(-t^2/2)

Same API and numbers as the reference's ``fdwt/cwt.py``: ``cwt``, ``CWT1D``, ``MorletPlan``,
``freqs_to_scales``, ``scales_to_freqs``, the fused consumers ``morlet_mix`` and
``spectral_softmax``, and the private names tests touch (``_apply_plan``,
``_MorletMixFunction.MIX_CHUNK_BYTES``, ``_SpectralSoftmaxFunction.CHUNK_BYTES``).

``method="fast"`` (octave pyramid) and ``"direct"`` (one octave, exact supports) run the
row-resident pyramid kernels of ``libfdwt_b200.so`` (``fdwt_cwt_forward`` & co. in
``include/fdwt_b200.h``): one launch computes every octave, the half-band chain stays in shared
memory, and the mixers never write the scalogram.  ``method="fft"`` applies the same filters
through cuFFT (``torch.fft``), as the reference does.  Inputs must be CUDA tensors.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from functools import lru_cache
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
from torch import nn

from . import _lib

__all__ = ["cwt", "CWT1D", "MorletPlan", "freqs_to_scales", "scales_to_freqs", "morlet_mix",
           "morlet_mix_tokens", "spectral_softmax"]

_PI_M14 = math.pi ** -0.25
_MAX_OCT, _MAX_SCALES, _MAX_LP = 24, 256, 49


def freqs_to_scales(freqs, fs: float = 1.0, w0: float = 6.0) -> torch.Tensor:
    """Morlet scale, in samples, whose centre frequency is ``freqs`` (in the unit of ``fs``):
    ``w0 fs / (2 pi f)``, as fp64."""
    f = torch.as_tensor(freqs, dtype=torch.float64)
    return w0 * fs / (2 * math.pi * f)


def scales_to_freqs(scales, fs: float = 1.0, w0: float = 6.0) -> torch.Tensor:
    """Inverse of :func:`freqs_to_scales` (the same expression with the roles swapped)."""
    s = torch.as_tensor(scales, dtype=torch.float64)
    return w0 * fs / (2 * math.pi * s)


def _halfband(c: int, beta: float) -> torch.Tensor:
    """The pyramid's anti-aliasing filter: 2c+1 taps of sinc(t/2) under a Kaiser window,
    scaled to unit DC gain (the reference designs the same filter, ``fdwt/cwt.py:65-68``)."""
    t = torch.arange(-c, c + 1, dtype=torch.float64)
    taps = torch.sinc(t / 2) * torch.from_numpy(np.kaiser(2 * c + 1, beta))
    return taps / taps.sum()


@dataclass
class _Stage:
    """The scales that share one octave of the pyramid."""
    octave: int
    dil: int                # tap spacing 2**octave in samples of x
    scale_idx: List[int]    # the scales' user indices, in increasing support
    half: int               # the octave's filters span taps -half .. half
    support: List[int]      # half-support (in taps) of each scale, same order


def _octave_of(scale: float, s_th: float, pyramid: bool) -> int:
    """Octave that computes ``scale``: the largest j >= 0 with 2^j s_th <= scale (0 unless
    the transform runs on the pyramid)."""
    if not pyramid:
        return 0
    return max(0, math.floor(math.log2(scale / s_th)))


def _support_taps(scale: float, reach: float, dil: int) -> int:
    """Half-support in taps of spacing ``dil``: the Gaussian envelope is cut at ``reach``
    scale units (at least one tap)."""
    return max(1, math.ceil(reach * scale / dil))


class _PlanC(ctypes.Structure):
    """ctypes mirror of ``fdwt_morlet_plan`` (include/fdwt_b200.h)."""

    _fields_ = [("n_octaves", ctypes.c_int32), ("n_scales", ctypes.c_int32),
                ("channels", ctypes.c_int32), ("center", ctypes.c_int32),
                ("c_lp", ctypes.c_int32),
                ("margins", ctypes.c_int32 * _MAX_OCT), ("oct_half", ctypes.c_int32 * _MAX_OCT),
                ("oct_begin", ctypes.c_int32 * _MAX_OCT), ("oct_count", ctypes.c_int32 * _MAX_OCT),
                ("order", ctypes.c_int32 * _MAX_SCALES), ("support", ctypes.c_int32 * _MAX_SCALES),
                ("lowpass", ctypes.c_double * _MAX_LP)]


class MorletPlan:
    """What a Morlet CWT needs besides the signal: the octave of each scale, the filter
    supports and the pyramid margins.  It depends on the initial scales only, so learnable
    scales reuse one plan while :meth:`filters` resamples the current ones.

    The rules are the reference's (``fdwt/cwt.py:80-203``), restated:
    - ``s_th = (w0 + truncate) / (0.8 pi)``; with ``method="fast"`` octave j takes the scales
      in ``[2^j s_th, 2^(j+1) s_th)`` (their band stays under 0.8 pi after j half-band steps),
      otherwise every scale is in octave 0;
    - a scale's half-support is ``ceil(truncate * support_margin * s / 2^j)`` taps;
    - the half-band filter has 33 taps (Kaiser beta 8), or 49 (beta 10) when ``truncate > 4.5``;
    - ``x_j`` (j >= 1) is kept on ``[-m_j, N + m_j)``: ``m_j`` covers octave j's own reach and
      that of the half-band steps feeding the coarser octaves.
    """

    def __init__(self, scales: Sequence[float], w0: float = 6.0, truncate: float = 4.0,
                 norm: str = "l2", complex: bool = True, method: str = "fast",
                 support_margin: float = 1.0):
        if method not in ("fast", "direct", "fft"):
            raise ValueError(f"unknown method '{method}' (expected 'fast', 'direct' or 'fft')")
        if norm not in ("l1", "l2"):
            raise ValueError("norm must be 'l1' or 'l2'")
        values = [float(v) for v in scales]
        if len(values) == 0 or min(values) <= 0:
            raise ValueError("scales must be a non-empty sequence of positive numbers")
        self.scales = values
        self.w0, self.truncate, self.norm = float(w0), float(truncate), norm
        self.complex, self.method = bool(complex), method
        self.channels = 2 if self.complex else 1
        self.s_th = (w0 + truncate) / (0.8 * math.pi)
        reach = truncate * support_margin

        octave = [_octave_of(v, self.s_th, method == "fast") for v in values]
        self.stages: List[_Stage] = []
        for j in sorted(set(octave)):
            dil = 1 << j
            members = [i for i, o in enumerate(octave) if o == j]
            taps = {i: _support_taps(values[i], reach, dil) for i in members}
            members.sort(key=taps.__getitem__)  # stable: equal supports keep the user's order
            supports = [taps[i] for i in members]
            self.stages.append(_Stage(j, dil, members, max(supports), supports))
        self.n_octaves = self.stages[-1].octave + 1
        self.center = max(st.half for st in self.stages)
        # per user scale: its tap spacing and half-support (the filters' sampling grid)
        self._dil = [0.0] * len(values)
        self._sup = [0.0] * len(values)
        for st in self.stages:
            for i, c in zip(st.scale_idx, st.support):
                self._dil[i] = float(st.dil)
                self._sup[i] = float(c)

        pyramid = self.n_octaves > 1
        c_lp, beta = (16, 8.0) if truncate <= 4.5 else (24, 10.0)
        self.c_lp = c_lp if pyramid else 0
        self.lowpass = _halfband(c_lp, beta) if pyramid else torch.zeros(1, dtype=torch.float64)

        # margins, coarse to fine: octave j's own filter reach, or what the half-band step
        # into x_{j+1} needs to leave x_{j+1}'s margin exact, whichever is larger
        last = self.n_octaves - 1
        reach_of = {st.octave: st.half * st.dil for st in self.stages}
        self.margins = [0] * (last + 1)
        for j in range(last, 0, -1):
            feed = self.margins[j + 1] + self.c_lp * (1 << j) if j < last else 0
            self.margins[j] = max(reach_of.get(j, 0), feed)
        self._static_cache: Dict = {}
        self._capi_struct = None

    @property
    def num_scales(self) -> int:
        return len(self.scales)

    def halfband_taps(self, device, dtype) -> torch.Tensor:
        """The half-band taps from the centre out, ``lowpass[c_lp + t]`` for t = 0..c_lp (the
        reference exposes the same accessor)."""
        key = ("hb", torch.device(device), dtype)
        if key not in self._static_cache:
            self._static_cache[key] = self.lowpass[self.c_lp:].to(device=device, dtype=dtype)
        return self._static_cache[key]

    def filters(self, scales: torch.Tensor, w0, dtype: torch.dtype) -> torch.Tensor:
        """Every sampled filter in one ``(S*C, 2*center+1)`` tensor, row ``i*C + c`` (c = 0 the
        real part, 1 the imaginary part), centre tap at column ``center``.

        Scale i is sampled at its octave's tap spacing d: tap k sits at ``u = k d / s`` scale
        units, and its value is ``pi^(-1/4) (d / n(s)) (e^{i w0 u} - e^{-w0^2/2}) e^{-u^2/2}``
        inside the scale's support and 0 outside, n(s) = sqrt(s) for the l2 norm, s for l1 (the
        factor d makes the dilated sum a Riemann sum of spacing d).  Differentiable in
        ``scales`` and in ``w0`` when it is a tensor; computed in fp64.
        """
        f64 = torch.float64
        dev = scales.device
        s = scales.to(f64).unsqueeze(1)
        spacing = torch.tensor(self._dil, dtype=f64, device=dev).unsqueeze(1)
        limit = torch.tensor(self._sup, dtype=f64, device=dev).unsqueeze(1)
        k = torch.arange(-self.center, self.center + 1, dtype=f64, device=dev).unsqueeze(0)
        u = k * spacing / s
        window = torch.exp(-0.5 * u * u) * (k.abs() <= limit)
        gain = _PI_M14 * spacing / (s.sqrt() if self.norm == "l2" else s)
        wave = torch.as_tensor(w0, dtype=f64, device=dev)
        phase = wave * u
        real = (torch.cos(phase) - torch.exp(-0.5 * wave * wave)) * window * gain
        if not self.complex:
            return real.to(dtype)
        imag = torch.sin(phase) * window * gain
        return torch.stack((real, imag), dim=1).reshape(-1, k.shape[1]).to(dtype)

    def capi(self) -> _PlanC:
        """The plan as the C struct the kernels take (built once)."""
        if self._capi_struct is None:
            if self.n_octaves > _MAX_OCT or self.num_scales > _MAX_SCALES:
                raise ValueError(f"the sm_100a kernels support up to {_MAX_OCT} octaves and "
                                 f"{_MAX_SCALES} scales")
            c = _PlanC()
            c.n_octaves, c.n_scales = self.n_octaves, self.num_scales
            c.channels, c.center, c.c_lp = self.channels, self.center, self.c_lp
            for j, m in enumerate(self.margins):
                c.margins[j] = m
            k = 0
            for st in self.stages:
                c.oct_half[st.octave] = st.half
                c.oct_begin[st.octave] = k
                c.oct_count[st.octave] = len(st.scale_idx)
                for i, sup in zip(st.scale_idx, st.support):
                    c.order[k], c.support[k] = i, sup
                    k += 1
            lp = self.lowpass.tolist()
            for t, v in enumerate(lp[:_MAX_LP]):
                c.lowpass[t] = v
            self._capi_struct = c
        return self._capi_struct


# --------------------------------------------------------------------------- kernel calls


def _out_dtype(dtype: torch.dtype) -> torch.dtype:
    return torch.float64 if dtype == torch.float64 else torch.float32


def _filters_on(H: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    return H.detach().to(device=x.device, dtype=x.dtype).contiguous()


def _cwt_forward(x: torch.Tensor, plan: MorletPlan, H: torch.Tensor) -> torch.Tensor:
    """Rows ``x (R, N)`` (fp32/fp64) -> ``y (R, S, N, C)``."""
    dev = _lib.require_cuda(x, H)
    lib = _lib.load()
    R, N = x.shape
    y = torch.empty((R, plan.num_scales, N, plan.channels), device=dev, dtype=x.dtype)
    Hd = _filters_on(H, x)
    with torch.cuda.device(dev):
        st = lib.fdwt_cwt_forward(_lib.dtype_code(x.dtype), R, N, x.data_ptr(), Hd.data_ptr(),
                                  ctypes.addressof(plan.capi()), y.data_ptr(), _lib.stream_of(dev))
    _lib.check(st, "fdwt_cwt_forward")
    return y


def _placeholder(like: torch.Tensor) -> torch.Tensor:
    return like.new_zeros(0)


def _cwt_backward(g: torch.Tensor, x: torch.Tensor, plan: MorletPlan, H: torch.Tensor,
                  need_x: bool, need_h: bool):
    """``(dL/dx (R, N), dL/dH (S*C, 2*center+1))`` from ``dL/dW (R, S, N, C)``: the adjoint
    chain and the filter gradient in one kernel (plus the row reduction of dL/dH)."""
    dev = _lib.require_cuda(g, x, H)
    lib = _lib.load()
    g = g.contiguous()
    R, _, N, _ = g.shape
    dt = g.dtype
    Hd = _filters_on(H, g)
    gx = torch.empty((R, N), device=dev, dtype=dt) if need_x else None
    gh = torch.empty_like(Hd) if need_h else None
    xd = x.detach().to(dt).contiguous() if need_h else None
    code = _lib.dtype_code(dt)
    with torch.cuda.device(dev):
        nws = lib.fdwt_cwt_backward_workspace(code, R, N, ctypes.addressof(plan.capi()),
                                              int(need_h))
        ws = _lib.workspace(nws, dev)
        st = lib.fdwt_cwt_backward(
            code, R, N, None if xd is None else xd.data_ptr(), Hd.data_ptr(),
            ctypes.addressof(plan.capi()), g.data_ptr(), None if gx is None else gx.data_ptr(),
            None if gh is None else gh.data_ptr(), None if ws is None else ws.data_ptr(), nws,
            _lib.stream_of(dev))
    _lib.check(st, "fdwt_cwt_backward")
    return gx, gh


class _MorletCWTFunction(torch.autograd.Function):
    """All octaves of the transform in one autograd node (``fdwt/cwt.py:213-281``)."""

    @staticmethod
    def forward(ctx, x, plan: MorletPlan, H):
        ctx.plan = plan
        ctx.save_for_backward(x, H)
        return _cwt_forward(x, plan, H)

    @staticmethod
    def backward(ctx, g):
        x, H = ctx.saved_tensors
        need_x, need_h = ctx.needs_input_grad[0], ctx.needs_input_grad[2]
        if not (need_x or need_h):
            return None, None, None
        gx, gH = _CWTBackwardFunction.apply(g, x, ctx.plan, H, need_x, need_h)
        return (gx if need_x else None), None, (gH.to(H.dtype) if need_h else None)


class _CWTBackwardFunction(torch.autograd.Function):
    """``(gx, gH) = (M_H^T g, dL/dH)`` of the transform.

    ``gx`` is linear in ``g`` and ``gH`` bilinear in ``(x, g)``, so the derivatives of this node
    are again the transform and these two outputs with other operands:
    ``d/dg = M_H ggx + M_ggH x``, ``d/dx = M_ggH^T g``, ``d/dH = dL/dH(x = ggx, g)``.  The
    transform therefore has derivatives of every order.
    """

    @staticmethod
    def forward(ctx, g, x, plan: MorletPlan, H, need_x: bool, need_h: bool):
        gx, gh = _cwt_backward(g, x, plan, H, need_x, need_h)
        ctx.plan, ctx.flags = plan, (need_x, need_h)
        ctx.save_for_backward(g, x, H)
        gx = _placeholder(g) if gx is None else gx
        gh = _placeholder(g) if gh is None else gh
        return gx, gh

    @staticmethod
    def backward(ctx, ggx, ggH):
        g, x, H = ctx.saved_tensors
        plan = ctx.plan
        need_x, need_h = ctx.flags
        ggx = ggx if (need_x and ggx is not None) else None
        ggH = ggH if (need_h and ggH is not None) else None
        gg = gx2 = gH2 = None
        if ctx.needs_input_grad[0]:
            if ggx is not None:
                gg = _MorletCWTFunction.apply(ggx, plan, H)
            if ggH is not None:
                t = _MorletCWTFunction.apply(x.to(g.dtype), plan, ggH)
                gg = t if gg is None else gg + t
        if ctx.needs_input_grad[1] and ggH is not None:
            gx2, _ = _CWTBackwardFunction.apply(g, x, plan, ggH, True, False)
        if ctx.needs_input_grad[3] and ggx is not None:
            _, gH2 = _CWTBackwardFunction.apply(g, ggx, plan, H, False, True)
            gH2 = gH2.to(H.dtype)
        return gg, gx2, None, gH2, None, None


def _fft_transform(x: torch.Tensor, plan: MorletPlan, H: torch.Tensor) -> torch.Tensor:
    """``method="fft"``: the direct filters applied through cuFFT (``fdwt/cwt.py:586-594``)."""
    R, N = x.shape
    C = plan.channels
    out = x.new_zeros((R, plan.num_scales, N, C))
    for st in plan.stages:
        rows = [i * C + c for i in st.scale_idx for c in range(C)]
        h = H[rows][:, plan.center - st.half: plan.center + st.half + 1].to(x.dtype)
        K = h.shape[1]
        nfft = 1 << (N + K - 1 - 1).bit_length()
        X = torch.fft.rfft(x, nfft)
        Hf = torch.fft.rfft(h, nfft)
        y = torch.fft.irfft(X[:, None, :] * Hf[None], nfft)[..., st.half:st.half + N]
        y = y.reshape(R, len(st.scale_idx), C, N).transpose(-1, -2)
        out = out.index_copy(1, torch.tensor(st.scale_idx, device=x.device), y)
    return out


def _apply_plan(x: torch.Tensor, plan: MorletPlan, H: torch.Tensor) -> torch.Tensor:
    """``x (..., N)`` -> ``(..., S, N)`` complex (real if ``plan.complex`` is False)."""
    if not x.is_floating_point() or x.is_complex():
        raise TypeError("cwt expects a real floating point tensor")
    _lib.require_cuda(x)
    lead, N = x.shape[:-1], x.shape[-1]
    x2 = x.reshape(-1, N).contiguous()
    if x2.dtype not in (torch.float32, torch.float64):
        x2 = x2.float()
    if plan.method == "fft":
        y = _fft_transform(x2, plan, H.to(x2.dtype))
    else:
        y = _MorletCWTFunction.apply(x2, plan, H)
    y = y.reshape(*lead, plan.num_scales, N, plan.channels)
    return torch.view_as_complex(y) if plan.complex else y[..., 0]


@lru_cache(maxsize=64)
def _cached_plan(scales: Tuple[float, ...], w0, truncate, norm, complex, method) -> MorletPlan:
    """Plans of the functional :func:`cwt`, shared between calls with the same arguments."""
    return MorletPlan(scales, w0, truncate, norm, complex, method)


@lru_cache(maxsize=64)
def _cached_filters(plan: MorletPlan, device: torch.device, dtype: torch.dtype):
    """The fixed filters of a cached plan on one device, in one dtype."""
    return plan.filters(torch.tensor(plan.scales, dtype=torch.float64, device=device), plan.w0,
                        dtype)


def _resolve_scales(scales, freqs, fs, w0) -> List[float]:
    """The scales in samples from exactly one of ``scales`` / ``freqs`` (with ``fs``, ``w0``)."""
    if (scales is None) == (freqs is None):
        raise ValueError("pass exactly one of `scales` or `freqs`")
    if freqs is not None:
        values = freqs_to_scales(freqs, fs, w0)
    else:
        values = torch.as_tensor(scales, dtype=torch.float64)
    return values.flatten().tolist()


def _compute_dtype(x: torch.Tensor) -> torch.dtype:
    return torch.float64 if x.dtype == torch.float64 else torch.float32


def cwt(x: torch.Tensor, scales: Optional[Sequence[float]] = None, *, freqs=None, fs: float = 1.0,
        w0: float = 6.0, method: str = "fast", norm: str = "l2", complex: bool = True,
        truncate: float = 4.0) -> torch.Tensor:
    """Morlet CWT of the real rows ``x (..., N)``: ``(..., S, N)``, complex unless
    ``complex=False``.  Give the scales in samples (``scales``) or as centre frequencies in
    the unit of ``fs`` (``freqs``, ``scale = w0 fs / (2 pi f)``); ``method`` is ``"fast"``
    (octave pyramid), ``"direct"`` (every scale at full rate) or ``"fft"``."""
    plan = _cached_plan(tuple(_resolve_scales(scales, freqs, fs, w0)), float(w0),
                        float(truncate), norm, bool(complex), method)
    return _apply_plan(x, plan, _cached_filters(plan, x.device, _compute_dtype(x)))


class CWT1D(nn.Module):
    """The Morlet CWT as a module (the reference's ``CWT1D``, ``fdwt/cwt.py:654-716``): real
    ``(..., N)`` in, ``(..., S, N)`` complex out (real with ``complex=False``).

    ``learnable=True`` makes the log-scales a parameter (``log_scales``, fp32) and
    ``learnable_w0=True`` the wave number (``w0``); gradients reach them through the
    filter-gradient kernels.  Otherwise ``log_scales`` is a buffer, ``w0`` a float, and the
    sampled filters are cached per device and dtype.  ``support_margin`` (default 1.25 when
    learning, else 1) widens the filter supports so that scales can grow.
    """

    def __init__(self, freqs=None, scales=None, fs: float = 1.0, w0: float = 6.0,
                 method: str = "fast", norm: str = "l2", complex: bool = True,
                 truncate: float = 4.0, learnable: bool = False, learnable_w0: bool = False,
                 support_margin: Optional[float] = None):
        super().__init__()
        values = _resolve_scales(scales, freqs, fs, w0)
        margin = support_margin if support_margin is not None else (1.25 if learnable else 1.0)
        self.fs = fs
        self.plan = MorletPlan(values, w0, truncate, norm, complex, method, margin)
        log_scales = torch.tensor(values, dtype=torch.float64).log().float()
        if learnable:
            self.log_scales = nn.Parameter(log_scales)
        else:
            self.register_buffer("log_scales", log_scales)
        self.w0 = nn.Parameter(torch.tensor(float(w0))) if learnable_w0 else float(w0)
        self._learn = bool(learnable or learnable_w0)
        self._filter_cache: Dict = {}

    @property
    def scales(self) -> torch.Tensor:
        """Current scales in samples."""
        return torch.exp(self.log_scales)

    @property
    def w0_value(self) -> float:
        w = self.w0
        return float(w.detach()) if isinstance(w, torch.Tensor) else float(w)

    @property
    def freqs(self) -> torch.Tensor:
        """Current centre frequencies in the unit of ``fs``."""
        return scales_to_freqs(self.scales.detach(), self.fs, self.w0_value)

    def _filters(self, device, dtype):
        if self._learn:  # rebuilt every call: the graph runs back to log_scales / w0
            return self.plan.filters(torch.exp(self.log_scales.to(torch.float64)), self.w0,
                                     dtype)
        key = (device, dtype)
        cached = self._filter_cache.get(key)
        if cached is None:
            cached = self.plan.filters(self.scales.to(torch.float64), self.w0, dtype)
            self._filter_cache = {key: cached}
        return cached

    def _apply(self, fn, *args, **kwargs):
        self._filter_cache = {}  # moved or cast: the cached filters are stale
        return super()._apply(fn, *args, **kwargs)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _apply_plan(x, self.plan, self._filters(x.device, _compute_dtype(x)))

    def extra_repr(self) -> str:
        p = self.plan
        return (f"scales={p.num_scales}, w0={self.w0_value:g}, method={p.method}, norm={p.norm}, "
                f"complex={p.complex}, octaves={p.n_octaves}, learnable={self._learn}")


# --------------------------------------------------------------------------- fused consumers
#
# Higher-order derivatives.  The fused kernels' backward passes return first derivatives only.
# When a backward runs with create_graph=True, the two consumers below instead recompute their
# output through the transform node (whose derivatives of every order come from the forward,
# adjoint and filter-gradient kernels) followed by the consumer written with torch ops, and take
# the gradient of that graph with create_graph=True: the scalogram is materialised for that
# call only.  The reference's CPU path gets the same derivatives from autograd
# (fdwt/cwt.py:391-394, 545-549).


def _scalogram_magnitude(W: torch.Tensor, plan: "MorletPlan") -> torch.Tensor:
    """``|W|`` of a ``(R, S, N, C)`` transform output, as torch's complex ``abs``."""
    if plan.channels == 2:
        return torch.view_as_complex(W).abs()
    return W[..., 0].abs()


def _mix_composed(x, plan, H, a, b):
    """``sum_s a[d, s] |W_s| + b[d, s] Re W_s`` on rows ``x (R, N)`` through the transform node."""
    W = _MorletCWTFunction.apply(x, plan, H)
    R, S, N, _ = W.shape
    D = a.shape[0]
    mag = _scalogram_magnitude(W, plan).view(R // D, D, S, N)
    re = W[..., 0].view(R // D, D, S, N)
    y = torch.einsum("bdsn,ds->bdn", mag, a.to(W.dtype)) + \
        torch.einsum("bdsn,ds->bdn", re, b.to(W.dtype))
    return y.reshape(R, N)


def _softmax_composed(x, plan, H, V, nch, tau):
    """``sum_f softmax_f(|W_f| / tau) V_f`` on rows ``x (R, N)`` through the transform node."""
    W = _MorletCWTFunction.apply(x, plan, H)
    R = W.shape[0]
    p = torch.softmax(_scalogram_magnitude(W, plan) / tau, dim=1)  # (R, S, N)
    Vd = V.to(W.dtype)
    Vr = Vd.repeat(R // nch, 1)[:, :, None] if Vd.dim() == 2 else \
        Vd.repeat_interleave(nch, dim=0)
    return (p * Vr).sum(1)


def _recomputed_grads(ctx, gy, inputs, fn, slots):
    """Gradients of ``fn(*inputs)`` against ``gy`` with create_graph=True, placed in the
    Function's argument slots ``slots`` (the other slots get None)."""
    needs = [ctx.needs_input_grad[k] for k in slots]
    with torch.enable_grad():
        y = fn(*inputs)
        wrt = [t for t, n in zip(inputs, needs) if n]
        grads = iter(torch.autograd.grad(y, wrt, gy, create_graph=True, allow_unused=True)
                     if wrt else [])
    out = [None] * (max(slots) + 1)
    for k, t, n in zip(slots, inputs, needs):
        if n:
            g = next(grads)
            out[k] = torch.zeros_like(t) if g is None else g.to(t.dtype)
    return tuple(out)



def _mix_forward(x2, plan, H, a, b):
    dev = _lib.require_cuda(x2, H, a, b)
    lib = _lib.load()
    R, N = x2.shape
    y = torch.empty((R, N), device=dev, dtype=x2.dtype)
    Hd = _filters_on(H, x2)
    a_ = a.detach().to(x2.dtype).contiguous()
    b_ = b.detach().to(x2.dtype).contiguous()
    with torch.cuda.device(dev):
        st = lib.fdwt_mix_forward(_lib.dtype_code(x2.dtype), R, N, x2.data_ptr(), Hd.data_ptr(),
                                  ctypes.addressof(plan.capi()), a_.data_ptr(), b_.data_ptr(),
                                  a_.shape[0], y.data_ptr(), _lib.stream_of(dev))
    _lib.check(st, "fdwt_mix_forward")
    return y


def _mix_backward(gy, x, plan, H, a, b, need_x, need_h):
    dev = _lib.require_cuda(gy, x, H, a, b)
    lib = _lib.load()
    R, N = x.shape
    dt = x.dtype
    gy = gy.to(dt).contiguous()
    Hd = _filters_on(H, x)
    a_ = a.detach().to(dt).contiguous()
    b_ = b.detach().to(dt).contiguous()
    D = a_.shape[0]
    gx = torch.empty((R, N), device=dev, dtype=dt) if need_x else None
    gh = torch.empty_like(Hd) if need_h else None
    ga = torch.empty_like(a_)
    gb = torch.empty_like(b_)
    code = _lib.dtype_code(dt)
    plan_p = ctypes.addressof(plan.capi())
    with torch.cuda.device(dev):
        nws = lib.fdwt_mix_backward_workspace(code, R, N, plan_p, D, int(need_h))
        ws = _lib.workspace(nws, dev)
        st = lib.fdwt_mix_backward(
            code, R, N, x.data_ptr(), Hd.data_ptr(), plan_p, a_.data_ptr(), b_.data_ptr(), D,
            gy.data_ptr(), None if gx is None else gx.data_ptr(),
            None if gh is None else gh.data_ptr(), ga.data_ptr(), gb.data_ptr(),
            None if ws is None else ws.data_ptr(), nws, _lib.stream_of(dev))
    _lib.check(st, "fdwt_mix_backward")
    return gx, gh, ga, gb


class _MorletMixFunction(torch.autograd.Function):
    """``y[r, n] = sum_s a[d, s] |W_s[r, n]| + b[d, s] Re W_s[r, n]`` without materialising W
    (``fdwt/cwt.py:284-376``).  ``MIX_CHUNK_BYTES`` is kept for drop-in compatibility; the
    sm_100a backward recomputes per row and needs no row chunking."""

    MIX_CHUNK_BYTES = 256 * 2**20

    @staticmethod
    def forward(ctx, x, plan: MorletPlan, H, a, b):
        ctx.plan = plan
        ctx.save_for_backward(x, H, a, b)
        return _mix_forward(x, plan, H, a, b)

    @staticmethod
    def backward(ctx, gy):
        x, H, a, b = ctx.saved_tensors
        if torch.is_grad_enabled():  # create_graph: gradients that are differentiable again
            return _recomputed_grads(ctx, gy, (x, H, a, b), lambda x_, H_, a_, b_: _mix_composed(
                x_, ctx.plan, H_, a_, b_), (0, 2, 3, 4))
        need_h = ctx.needs_input_grad[2]
        gx, gH, ga, gb = _mix_backward(gy, x, ctx.plan, H, a, b, ctx.needs_input_grad[0],
                                       need_h)
        return (gx, None, gH.to(H.dtype) if need_h else None, ga.to(a.dtype), gb.to(b.dtype))


def morlet_mix(x: torch.Tensor, plan: MorletPlan, H: torch.Tensor, a: torch.Tensor,
               b: torch.Tensor) -> torch.Tensor:
    """``x (B, D, N)`` -> ``sum_s a[d, s] |W_s| + b[d, s] Re W_s``, shape ``(B, D, N)``."""
    B, D, N = x.shape
    _lib.require_cuda(x)
    x2 = x.reshape(B * D, N).contiguous()
    if x2.dtype not in (torch.float32, torch.float64):
        x2 = x2.float()
    return _MorletMixFunction.apply(x2, plan, H, a, b).view(B, D, N)


def _mix_tokens_forward(x, plan, H, a, b, bias):
    dev = _lib.require_cuda(x, H, a, b)
    lib = _lib.load()
    B, N, D = x.shape
    y = torch.empty_like(x)
    Hd = _filters_on(H, x)
    a_ = a.detach().to(x.dtype).contiguous()
    b_ = b.detach().to(x.dtype).contiguous()
    c_ = None if bias is None else bias.detach().to(x.dtype).contiguous()
    with torch.cuda.device(dev):
        st = lib.fdwt_mix_tokens_forward(
            _lib.dtype_code(x.dtype), B, N, D, x.data_ptr(), Hd.data_ptr(),
            ctypes.addressof(plan.capi()), a_.data_ptr(), b_.data_ptr(),
            None if c_ is None else c_.data_ptr(), y.data_ptr(), _lib.stream_of(dev))
    _lib.check(st, "fdwt_mix_tokens_forward")
    return y


def _mix_tokens_backward(gy, x, plan, H, a, b, need_x, need_h, need_bias):
    dev = _lib.require_cuda(gy, x, H, a, b)
    lib = _lib.load()
    B, N, D = x.shape
    dt = x.dtype
    gy = gy.to(dt).contiguous()
    Hd = _filters_on(H, x)
    a_ = a.detach().to(dt).contiguous()
    b_ = b.detach().to(dt).contiguous()
    gx = torch.empty_like(x) if need_x else None
    gh = torch.empty_like(Hd) if need_h else None
    ga = torch.empty_like(a_)
    gb = torch.empty_like(b_)
    gc = torch.empty(D, device=dev, dtype=dt) if need_bias else None
    code = _lib.dtype_code(dt)
    plan_p = ctypes.addressof(plan.capi())
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    with torch.cuda.device(dev):
        nws = lib.fdwt_mix_tokens_backward_workspace(code, B, N, D, plan_p, int(need_h))
        ws = _lib.workspace(nws, dev)
        st = lib.fdwt_mix_tokens_backward(
            code, B, N, D, x.data_ptr(), Hd.data_ptr(), plan_p, a_.data_ptr(), b_.data_ptr(),
            gy.data_ptr(), ptr(gx), ptr(gh), ga.data_ptr(), gb.data_ptr(), ptr(gc), ptr(ws), nws,
            _lib.stream_of(dev))
    _lib.check(st, "fdwt_mix_tokens_backward")
    return gx, gh, ga, gb, gc


def _mix_tokens_composed(x, plan, H, a, b, bias):
    """The token-layout mix through the transform node (higher-order derivatives)."""
    B, N, D = x.shape
    y = _mix_composed(x.transpose(1, 2).reshape(B * D, N), plan, H, a, b)
    y = y.view(B, D, N).transpose(1, 2)
    return y if bias is None else y + bias.to(y.dtype)


class _MorletMixTokensFunction(torch.autograd.Function):
    """The mix on ``(B, N, D)`` tokens with the bias added: MorletTokenMixer's
    ``morlet_mix(x.transpose(1, 2), ...).transpose(1, 2) + bias`` (``fdwt/layers.py:49-55``)
    in one forward kernel and one backward call, without the transposes."""

    @staticmethod
    def forward(ctx, x, plan: MorletPlan, H, a, b, bias):
        ctx.plan = plan
        ctx.has_bias = bias is not None
        ctx.save_for_backward(x, H, a, b, bias if bias is not None else x.new_zeros(0))
        return _mix_tokens_forward(x, plan, H, a, b, bias)

    @staticmethod
    def backward(ctx, gy):
        x, H, a, b, bias = ctx.saved_tensors
        if not ctx.has_bias:
            bias = None
        if torch.is_grad_enabled():
            if bias is None:
                return _recomputed_grads(ctx, gy, (x, H, a, b), lambda x_, H_, a_, b_:
                                         _mix_tokens_composed(x_, ctx.plan, H_, a_, b_, None),
                                         (0, 2, 3, 4)) + (None,)
            return _recomputed_grads(ctx, gy, (x, H, a, b, bias), lambda x_, H_, a_, b_, c_:
                                     _mix_tokens_composed(x_, ctx.plan, H_, a_, b_, c_),
                                     (0, 2, 3, 4, 5))
        need_h = ctx.needs_input_grad[2]
        need_bias = bias is not None and ctx.needs_input_grad[5]
        gx, gH, ga, gb, gc = _mix_tokens_backward(gy, x, ctx.plan, H, a, b,
                                                  ctx.needs_input_grad[0], need_h, need_bias)
        return (gx, None, gH.to(H.dtype) if need_h else None, ga.to(a.dtype), gb.to(b.dtype),
                gc.to(bias.dtype) if need_bias else None)


def morlet_mix_tokens(x: torch.Tensor, plan: MorletPlan, H: torch.Tensor, a: torch.Tensor,
                      b: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x (B, N, D)`` -> ``sum_s a[d, s] |W_s x[b, :, d]| + b[d, s] Re W_s (+ bias[d])``,
    shape ``(B, N, D)``: ``morlet_mix`` on the token layout, read and written in place by the
    kernels (no transposes), with the bias added in the same kernel."""
    _lib.require_cuda(x)
    if x.dim() != 3:
        raise ValueError(f"expected (B, N, D) tokens, got shape {tuple(x.shape)}")
    dt = torch.float64 if x.dtype == torch.float64 else torch.float32
    xc = x if x.dtype == dt and x.is_contiguous() else x.to(dt).contiguous()
    return _MorletMixTokensFunction.apply(xc, plan, H, a, b, bias)


def _softmax_forward(x2, plan, H, V, nch, tau):
    dev = _lib.require_cuda(x2, H, V)
    lib = _lib.load()
    R, N = x2.shape
    out = torch.empty((R, N), device=dev, dtype=x2.dtype)
    m = torch.empty_like(out)
    l = torch.empty_like(out)
    Hd = _filters_on(H, x2)
    V_ = V.detach().to(x2.dtype).contiguous()
    with torch.cuda.device(dev):
        st = lib.fdwt_specsoftmax_forward(
            _lib.dtype_code(x2.dtype), R, N, x2.data_ptr(), Hd.data_ptr(),
            ctypes.addressof(plan.capi()), V_.data_ptr(), int(V_.dim() == 3), nch, 1.0 / tau,
            out.data_ptr(), m.data_ptr(), l.data_ptr(), _lib.stream_of(dev))
    _lib.check(st, "fdwt_specsoftmax_forward")
    return out, m, l


def _softmax_backward(gout, x, plan, H, V, nch, tau, m, l, out, need_x, need_h):
    dev = _lib.require_cuda(gout, x, H, V)
    lib = _lib.load()
    R, N = x.shape
    dt = x.dtype
    gout = gout.to(dt).contiguous()
    Hd = _filters_on(H, x)
    V_ = V.detach().to(dt).contiguous()
    v_pos = int(V_.dim() == 3)
    gx = torch.empty((R, N), device=dev, dtype=dt) if need_x else None
    gh = torch.empty_like(Hd) if need_h else None
    gv = torch.empty_like(V_)
    code = _lib.dtype_code(dt)
    plan_p = ctypes.addressof(plan.capi())
    with torch.cuda.device(dev):
        nws = lib.fdwt_specsoftmax_backward_workspace(code, R, N, plan_p, v_pos, nch,
                                                      int(need_h))
        ws = _lib.workspace(nws, dev)
        st = lib.fdwt_specsoftmax_backward(
            code, R, N, x.data_ptr(), Hd.data_ptr(), plan_p, V_.data_ptr(), v_pos, nch,
            1.0 / tau, m.data_ptr(), l.data_ptr(), out.data_ptr(), gout.data_ptr(),
            None if gx is None else gx.data_ptr(), None if gh is None else gh.data_ptr(),
            gv.data_ptr(), None if ws is None else ws.data_ptr(), nws, _lib.stream_of(dev))
    _lib.check(st, "fdwt_specsoftmax_backward")
    return gx, gh, gv


class _SpectralSoftmaxFunction(torch.autograd.Function):
    """``out[r, n] = sum_f softmax_f(|W_f x_r|(n) / tau) * V_f[r, n]`` without materialising W
    (``fdwt/cwt.py:397-509``).  ``CHUNK_BYTES`` is kept for drop-in compatibility."""

    CHUNK_BYTES = 256 * 2**20

    @staticmethod
    def forward(ctx, x, plan: MorletPlan, H, V, nch: int, tau: float, precision: str):
        if not plan.complex:
            raise ValueError("the spectral softmax needs the complex Morlet transform")
        out, m, l = _softmax_forward(x, plan, H, V, nch, tau)
        ctx.plan, ctx.nch, ctx.tau = plan, nch, tau
        ctx.save_for_backward(x, H, V, m, l, out)
        return out

    @staticmethod
    def backward(ctx, gy):
        x, H, V, m, l, out = ctx.saved_tensors
        if torch.is_grad_enabled():  # create_graph: gradients that are differentiable again
            return _recomputed_grads(
                ctx, gy, (x, H, V), lambda x_, H_, V_: _softmax_composed(
                    x_, ctx.plan, H_, V_, ctx.nch, ctx.tau), (0, 2, 3)) + (None, None, None)
        need_h = ctx.needs_input_grad[2]
        gx, gH, gV = _softmax_backward(gy, x, ctx.plan, H, V, ctx.nch, ctx.tau, m, l, out,
                                       ctx.needs_input_grad[0], need_h)
        return (gx, None, gH.to(H.dtype) if need_h else None, gV.to(V.dtype), None, None, None)


def spectral_softmax(x: torch.Tensor, plan: MorletPlan, H: torch.Tensor, V: torch.Tensor,
                     nch: int, tau: float = 1.0) -> torch.Tensor:
    """``x (R, N)`` -> ``sum_f softmax_f(|W_f x|/tau) V_f``, shape ``(R, N)``.

    ``V`` is ``(nch, S)`` (row r uses ``V[r % nch]``) or ``(R // nch, S, N)`` (row r uses
    ``V[r // nch]``).
    """
    R, N = x.shape
    _lib.require_cuda(x)
    x2 = x.contiguous()
    if x2.dtype not in (torch.float32, torch.float64):
        x2 = x2.float()
    return _SpectralSoftmaxFunction.apply(x2, plan, H, V, nch, float(tau), "ieee")
