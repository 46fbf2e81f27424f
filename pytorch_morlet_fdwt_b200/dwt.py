"""Fast (Mallat) discrete wavelet transform on sm_100a kernels.

Same API and numbers as the reference's ``fdwt/dwt.py`` (``dwt``, ``idwt``, ``wavedec``,
``waverec``, ``dwt_max_level``, ``DWT1D``, ``IDWT1D``): the transform acts on the last
dimension and every leading dimension is a batch dimension.

The reference launches one kernel per level from Python loops (``dwt.py:146-171``).  Here a
whole multilevel transform is ONE autograd node and one C-ABI call
(``fdwt_dwt_analysis`` / ``fdwt_dwt_synthesis`` in ``include/fdwt_b200.h``), which runs the
levels as a short chain of streaming launches:

* :class:`_AnalysisFn` -- multilevel analysis ``A``; its backward is :class:`_SynthesisFn`;
* :class:`_SynthesisFn` -- the exact transpose ``A^T``; its backward is :class:`_AnalysisFn`;
* :class:`_Analysis` / :class:`_Synthesis` -- the reference's per-level nodes with their
  ``apply`` signatures (``dwt.py:36-82``), each one single-level C-ABI call.

``wavedec`` is ``A`` with the ``dec_*`` filters; its gradient is ``A^T``.  ``idwt`` /
``waverec`` are ``A^T`` of a zero-mode (or periodization) analysis on the time-reversed
``rec_*`` filters, exactly as the reference defines them (``dwt.py:114-135``); pywt's trim rule
(``dwt.py:168-169``) is the transpose of appending a zero to an approximation.  Because the
two nodes are each other's backward, gradients of every order are available.
"""

from __future__ import annotations

import functools
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch
from torch import nn

from . import _lib, config
from .wavelets import WaveletLike, get_filter_bank

__all__ = ["dwt", "idwt", "wavedec", "waverec", "dwt_max_level", "dwt_coeff_len", "DWT1D",
           "IDWT1D", "MODES"]

MODES = {"zero": 0, "periodic": 1, "symmetric": 2, "reflect": 3, "periodization": 4}
_PERIODIZATION = MODES["periodization"]
_ZERO = MODES["zero"]


def _check_dtype(x: torch.Tensor):
    if not x.is_floating_point():
        raise TypeError(f"expected a floating point tensor, got {x.dtype}")


def _mode_id(mode: str) -> int:
    try:
        return MODES[mode]
    except KeyError:
        raise ValueError(f"unsupported mode '{mode}', expected one of {sorted(MODES)}") from None


def dwt_coeff_len(n: int, filter_len: int, mode: str) -> int:
    """Coefficient length of one level (``fdwt/dwt.py:97-100``)."""
    if mode == "periodization":
        return (n + 1) // 2
    return (n + filter_len - 1) // 2


def dwt_max_level(n: int, wavelet: WaveletLike = "db4") -> int:
    """Same as ``pywt.dwt_max_level``."""
    L = get_filter_bank(wavelet).length
    if L < 2 or n < L - 1:
        return 0
    return (n // (L - 1)).bit_length() - 1


@dataclass(frozen=True)
class _Spec:
    """A multilevel analysis operator: taps, boundary mode, offset and level lengths.

    ``coef_len[k]`` / ``pad[k]`` describe level ``k`` (finest first): the level maps a signal
    of length ``in_len[k]`` to coefficients of length ``coef_len[k]``, and the approximation
    handed to level ``k+1`` carries ``pad[k]`` extra trailing zeros.
    """

    h0: Tuple[float, ...]
    h1: Tuple[float, ...]
    mode: int
    off: int
    n: int
    coef_len: Tuple[int, ...]
    pad: Tuple[int, ...]

    @property
    def levels(self) -> int:
        return len(self.coef_len)

    @property
    def in_len(self) -> Tuple[int, ...]:
        return (self.n,) + tuple(c + p for c, p in zip(self.coef_len[:-1], self.pad[:-1]))

    @property
    def approx_len(self) -> int:
        return self.coef_len[-1] + self.pad[-1]


@functools.lru_cache(maxsize=512)
def _spec_arrays(spec: _Spec):
    """ctypes arrays of a spec's lengths and taps, built once per spec (the library only reads
    them): (coef_len, pad, h0, h1, in_len)."""
    return (_lib.i64_array(spec.coef_len), _lib.i64_array(spec.pad), _lib.f64_array(spec.h0),
            _lib.f64_array(spec.h1), _lib.i64_array(spec.in_len))


@functools.lru_cache(maxsize=1024)
def _analysis_ws(spec: _Spec, rows: int, dt: int, device_index: int) -> int:
    """Workspace bytes of an analysis call (a pure function of its sizes on one device: the
    query plans the launches, which costs host time worth saving on every call)."""
    coef, pad, _, _, _ = _spec_arrays(spec)
    return int(_lib.load().fdwt_dwt_analysis_workspace(dt, rows, spec.n, spec.levels, coef, pad,
                                                        len(spec.h0), spec.mode, spec.off))


@functools.lru_cache(maxsize=1024)
def _synthesis_ws(spec: _Spec, rows: int, dt: int, device_index: int) -> int:
    """Workspace bytes of a synthesis call (see _analysis_ws)."""
    coef, _, _, _, outl = _spec_arrays(spec)
    return int(_lib.load().fdwt_dwt_synthesis_workspace(dt, rows, spec.levels, spec.approx_len,
                                                         coef, outl, len(spec.h0), spec.mode,
                                                         spec.off))


def _rows(t: torch.Tensor, n: int) -> torch.Tensor:
    return t.reshape(-1, n).contiguous()


def _analysis(x: torch.Tensor, spec: _Spec) -> List[torch.Tensor]:
    """Kernel call: rows of ``x`` -> ``[approx, detail_J, ..., detail_1]``."""
    dev = _lib.require_cuda(x)
    lib = _lib.load()
    lead = x.shape[:-1]
    x2 = _rows(x, spec.n)
    R = x2.shape[0]
    outs = [torch.empty((R, spec.approx_len), device=dev, dtype=x.dtype)]
    outs += [torch.empty((R, c), device=dev, dtype=x.dtype) for c in reversed(spec.coef_len)]
    J, L = spec.levels, len(spec.h0)
    coef, pad, h0, h1, _ = _spec_arrays(spec)
    dt = _lib.dtype_code(x.dtype)
    with torch.cuda.device(dev):
        nws = _analysis_ws(spec, R, dt, dev.index)
        ws = _lib.workspace(nws, dev)
        st = lib.fdwt_dwt_analysis(
            dt, R, x2.data_ptr(), spec.n, J, coef, pad, _lib.ptr_array(outs),
            h0, h1, L, spec.mode, spec.off,
            None if ws is None else ws.data_ptr(), nws, _lib.stream_of(dev))
    _lib.check(st, "fdwt_dwt_analysis")
    if config.check_device_errors:
        _lib.check_device_error("fdwt_dwt_analysis")
    return [o.reshape(*lead, o.shape[-1]) for o in outs]


def _synthesis(inputs: Sequence[Optional[torch.Tensor]], spec: _Spec) -> torch.Tensor:
    """Kernel call: ``[approx, detail_J, ..., detail_1]`` -> rows of length ``spec.n``."""
    ref = next(t for t in inputs if t is not None)
    dev = _lib.require_cuda(*inputs)
    lib = _lib.load()
    lead = ref.shape[:-1]
    dtype = ref.dtype
    J, L = spec.levels, len(spec.h0)
    lens = [spec.approx_len] + list(reversed(spec.coef_len))
    rows = []
    for t, n in zip(inputs, lens):
        rows.append(None if t is None else _rows(t.to(dtype), n))
    R = ref.reshape(-1, ref.shape[-1]).shape[0]
    if rows[0] is None:
        rows[0] = torch.zeros((R, spec.approx_len), device=dev, dtype=dtype)
    y = torch.empty((R, spec.n), device=dev, dtype=dtype)
    coef, _, h0, h1, outl = _spec_arrays(spec)
    dt = _lib.dtype_code(dtype)
    with torch.cuda.device(dev):
        nws = _synthesis_ws(spec, R, dt, dev.index)
        ws = _lib.workspace(nws, dev)
        st = lib.fdwt_dwt_synthesis(
            dt, R, J, _lib.ptr_array(rows), spec.approx_len, coef, outl, y.data_ptr(),
            h0, h1, L, spec.mode, spec.off,
            None if ws is None else ws.data_ptr(), nws, _lib.stream_of(dev))
    _lib.check(st, "fdwt_dwt_synthesis")
    if config.check_device_errors:
        _lib.check_device_error("fdwt_dwt_synthesis")
    return y.reshape(*lead, spec.n)


class _AnalysisFn(torch.autograd.Function):
    """``(approx, d_J..d_1) = A x`` for a whole multilevel transform; backward = ``A^T``.

    The multilevel counterpart of :class:`_Analysis`: ``wavedec`` runs every level in one
    node (the reference chains one ``_Analysis`` per level, ``fdwt/dwt.py:146-158``)."""

    @staticmethod
    def forward(ctx, x, spec: _Spec):
        ctx.spec = spec
        ctx.set_materialize_grads(False)  # unused outputs reach the kernel as NULL (= zeros)
        return tuple(_analysis(x, spec))

    @staticmethod
    def backward(ctx, *grads):
        if all(g is None for g in grads):
            return None, None
        return _SynthesisFn.apply(ctx.spec, *grads), None


class _SynthesisFn(torch.autograd.Function):
    """``y = A^T (approx, d_J..d_1)``; backward = ``A``.

    The multilevel counterpart of :class:`_Synthesis`: ``waverec`` runs every level in one
    node (the reference chains one ``_Synthesis`` per level, ``fdwt/dwt.py:161-171``)."""

    @staticmethod
    def forward(ctx, spec: _Spec, *inputs):
        ctx.spec = spec
        ctx.set_materialize_grads(False)
        ctx.present = [t is not None for t in inputs]
        return _synthesis(inputs, spec)

    @staticmethod
    def backward(ctx, gy):
        if gy is None:
            return (None,) * (1 + len(ctx.present))
        grads = _AnalysisFn.apply(gy.contiguous(), ctx.spec)
        return (None,) + tuple(g if p else None for g, p in zip(grads, ctx.present))


def _taps(h: torch.Tensor) -> Tuple[float, ...]:
    """Filter taps of a 1-D tensor as the host doubles the C ABI takes."""
    return tuple(float(v) for v in h.detach().reshape(-1).double().cpu().tolist())


def _one_level_spec(h0, h1, mode: int, off: int, n: int, n_out: int) -> _Spec:
    if len(h0) != len(h1) or len(h0) % 2:
        raise ValueError("h0 and h1 must have the same even length")
    return _Spec(_taps(h0), _taps(h1), int(mode), int(off), int(n), (int(n_out),), (0,))


class _Analysis(torch.autograd.Function):
    """One level ``(y0, y1) = A x``; backward ``A^T`` through :class:`_Synthesis`.

    Same ``apply(x, h0, h1, mode, off, n_out)`` as the reference's per-level node
    (``fdwt/dwt.py:36-56``): ``h0``/``h1`` are the (even-length) filter tensors, ``mode`` the
    integer of ``MODES``, ``off`` the phase offset (1, or ``L // 2`` for periodization) and
    ``n_out`` the coefficient length.  One ``fdwt_dwt_analysis`` call with one level."""

    @staticmethod
    def forward(ctx, x, h0, h1, mode: int, off: int, n_out: int):
        spec = _one_level_spec(h0, h1, mode, off, x.shape[-1], n_out)
        ctx.save_for_backward(h0, h1)
        ctx.cfg = (mode, off, x.shape[-1])
        a, d = _analysis(x, spec)
        return a, d

    @staticmethod
    def backward(ctx, g0, g1):
        h0, h1 = ctx.saved_tensors
        mode, off, n = ctx.cfg
        gx = None
        if ctx.needs_input_grad[0] and (g0 is not None or g1 is not None):
            g0 = torch.zeros_like(g1) if g0 is None else g0
            g1 = torch.zeros_like(g0) if g1 is None else g1
            gx = _Synthesis.apply(g0, g1, h0, h1, mode, off, n)
        return gx, None, None, None, None, None


class _Synthesis(torch.autograd.Function):
    """One level ``y = A^T (a, d)``; backward ``A`` through :class:`_Analysis`.

    Same ``apply(a, d, h0, h1, mode, off, n)`` as the reference's per-level node
    (``fdwt/dwt.py:59-82``); ``n`` is the output length.  One ``fdwt_dwt_synthesis`` call with
    one level."""

    @staticmethod
    def forward(ctx, a, d, h0, h1, mode: int, off: int, n: int):
        if a.shape != d.shape:
            raise ValueError(f"cA and cD shapes differ: {tuple(a.shape)} vs {tuple(d.shape)}")
        spec = _one_level_spec(h0, h1, mode, off, n, a.shape[-1])
        ctx.save_for_backward(h0, h1)
        ctx.cfg = (mode, off, a.shape[-1])
        return _synthesis([a, d], spec)

    @staticmethod
    def backward(ctx, gy):
        h0, h1 = ctx.saved_tensors
        mode, off, nc = ctx.cfg
        ga = gd = None
        if gy is not None and (ctx.needs_input_grad[0] or ctx.needs_input_grad[1]):
            ga, gd = _Analysis.apply(gy, h0, h1, mode, off, nc)
        return ga, gd, None, None, None, None, None


def _bank(wavelet):
    return get_filter_bank(wavelet)


def _analysis_spec(bank, m: int, n: int, level: int, mode: str) -> _Spec:
    L = bank.length
    off = L // 2 if m == _PERIODIZATION else 1
    lens, cur = [], n
    for _ in range(level):
        if cur < 1:
            raise ValueError("the signal became empty before the requested level")
        cur = dwt_coeff_len(cur, L, mode)
        lens.append(cur)
    return _Spec(tuple(bank.dec_lo), tuple(bank.dec_hi), m, off, n, tuple(lens), (0,) * level)


def dwt(x: torch.Tensor, wavelet: WaveletLike = "db4", mode: str = "symmetric"
        ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Single level DWT along the last dimension. Returns ``(cA, cD)`` like ``pywt.dwt``."""
    _check_dtype(x)
    m = _mode_id(mode)
    bank = _bank(wavelet)
    if x.shape[-1] < 1:
        raise ValueError("the signal must have at least one sample")
    a, d = _AnalysisFn.apply(x, _analysis_spec(bank, m, x.shape[-1], 1, mode))
    return a, d


def _synthesis_len(m: int, nc: int, L: int) -> Tuple[int, int, int]:
    """(mode, off, n) of the analysis whose transpose is pywt's idwt (``dwt.py:127-135``)."""
    if m == _PERIODIZATION:
        return _PERIODIZATION, L // 2, 2 * nc
    n = 2 * nc - L + 2
    if n <= 0:
        raise ValueError(f"coefficients of length {nc} are too short for a filter of length {L}")
    return _ZERO, 1, n


def idwt(cA: Optional[torch.Tensor], cD: Optional[torch.Tensor], wavelet: WaveletLike = "db4",
         mode: str = "symmetric") -> torch.Tensor:
    """Single level inverse DWT, identical to ``pywt.idwt``."""
    if cA is None and cD is None:
        raise ValueError("at least one of cA, cD must be given")
    cA = torch.zeros_like(cD) if cA is None else cA
    cD = torch.zeros_like(cA) if cD is None else cD
    if cA.shape != cD.shape:
        raise ValueError(f"cA and cD shapes differ: {tuple(cA.shape)} vs {tuple(cD.shape)}")
    _check_dtype(cA)
    m = _mode_id(mode)
    bank = _bank(wavelet)
    L, nc = bank.length, cA.shape[-1]
    sm, off, n = _synthesis_len(m, nc, L)
    spec = _Spec(tuple(bank.rec_lo[::-1]), tuple(bank.rec_hi[::-1]), sm, off, n, (nc,), (0,))
    return _SynthesisFn.apply(spec, cA, cD)


def wavedec(x: torch.Tensor, wavelet: WaveletLike = "db4", mode: str = "symmetric",
            level: Optional[int] = None) -> List[torch.Tensor]:
    """Multilevel DWT: ``[cA_n, cD_n, ..., cD_1]`` exactly like ``pywt.wavedec``."""
    if level is None:
        level = dwt_max_level(x.shape[-1], wavelet)
    if level < 0:
        raise ValueError("level must be >= 0")
    if level == 0:
        return [x]
    _check_dtype(x)
    m = _mode_id(mode)
    bank = _bank(wavelet)
    if x.shape[-1] < 1:
        raise ValueError("the signal must have at least one sample")
    return list(_AnalysisFn.apply(x, _analysis_spec(bank, m, x.shape[-1], level, mode)))


def waverec(coeffs: Sequence[torch.Tensor], wavelet: WaveletLike = "db4",
            mode: str = "symmetric") -> torch.Tensor:
    """Inverse of :func:`wavedec`, like ``pywt.waverec`` (one fused launch for all levels)."""
    if len(coeffs) == 0:
        raise ValueError("coeffs must not be empty")
    a = coeffs[0]
    if len(coeffs) == 1:
        return a
    m = _mode_id(mode)
    bank = _bank(wavelet)
    L = bank.length
    details = list(coeffs[1:])
    for t in [a] + details:
        _check_dtype(t)
    # coarsest first: the incoming approximation may carry one extra sample (trimmed)
    a_len = a.shape[-1]
    lens, outs, pads = [], [], []
    sm = off = None
    for d in details:
        nc = d.shape[-1]
        if a_len == nc + 1:
            pads.append(1)
        elif a_len == nc:
            pads.append(0)
        else:
            raise ValueError(f"cA and cD shapes differ: {a_len} vs {nc} samples")
        if d.shape[:-1] != a.shape[:-1]:
            raise ValueError(f"cA and cD shapes differ: {tuple(a.shape)} vs {tuple(d.shape)}")
        sm, off, n = _synthesis_len(m, nc, L)
        lens.append(nc)
        outs.append(n)
        a_len = n
    # level k (finest first) pads its approximation by pads of the level above it
    coef_len = tuple(reversed(lens))
    pad = tuple(reversed(pads))
    spec = _Spec(tuple(bank.rec_lo[::-1]), tuple(bank.rec_hi[::-1]), sm, off, outs[-1],
                 coef_len, pad)
    return _SynthesisFn.apply(spec, a, *details)


class DWT1D(nn.Module):
    """Multilevel 1D DWT along the last dimension.

    ``forward(x)`` returns ``[cA_J, cD_J, ..., cD_1]`` (PyWavelets ordering).
    """

    def __init__(self, wavelet: WaveletLike = "db4", level: Optional[int] = None,
                 mode: str = "symmetric"):
        super().__init__()
        _mode_id(mode)
        self.bank = get_filter_bank(wavelet)
        self.level = level
        self.mode = mode

    def forward(self, x: torch.Tensor) -> List[torch.Tensor]:
        return wavedec(x, self.bank, self.mode, self.level)

    def extra_repr(self) -> str:
        return f"wavelet={self.bank.name}, level={self.level}, mode={self.mode}"


class IDWT1D(nn.Module):
    """Inverse of :class:`DWT1D`."""

    def __init__(self, wavelet: WaveletLike = "db4", mode: str = "symmetric"):
        super().__init__()
        _mode_id(mode)
        self.bank = get_filter_bank(wavelet)
        self.mode = mode

    def forward(self, coeffs: Sequence[torch.Tensor]) -> torch.Tensor:
        return waverec(coeffs, self.bank, self.mode)

    def extra_repr(self) -> str:
        return f"wavelet={self.bank.name}, mode={self.mode}"
