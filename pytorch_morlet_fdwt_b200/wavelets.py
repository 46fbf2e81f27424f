"""Two-channel filter banks for the discrete wavelet transform.

Mirrors the reference's ``fdwt/wavelets.py:18-90``: a frozen :class:`FilterBank` of
``dec_lo, dec_hi, rec_lo, rec_hi`` tuples padded to a common even length, resolved from a
name, a ``pywt.Wavelet``, a :class:`FilterBank` or a 4-sequence.

Named lookups use PyWavelets when it is importable (``wavelets.py:74-78``).  Without it,
``"haar"`` and ``"dbN"`` are still available: their coefficients are generated here by
Daubechies' spectral factorisation (minimum-phase root choice), which yields the PyWavelets
conventions ``rec_lo = h``, ``dec_lo = h[::-1]``, ``rec_hi[k] = (-1)^k h[L-1-k]``,
``dec_hi = rec_hi[::-1]``.  Every other name needs PyWavelets and raises ``ImportError``
as the reference does when it is missing.

The kernels take the taps by value (they land in the kernel's constant parameter bank), so
a bank is resolved to plain Python floats on the host and never round-trips the device.
"""

from __future__ import annotations

import re
from dataclasses import dataclass
from functools import lru_cache
from math import comb
from typing import Sequence, Union

import numpy as np
import torch

__all__ = ["FilterBank", "get_filter_bank", "WaveletLike", "daubechies_scaling_filter"]


@dataclass(frozen=True)
class FilterBank:
    """Analysis (``dec_*``) and synthesis (``rec_*``) filters of a two-channel filter bank."""

    name: str
    dec_lo: tuple
    dec_hi: tuple
    rec_lo: tuple
    rec_hi: tuple

    @property
    def length(self) -> int:
        return len(self.dec_lo)

    def tensors(self, device, dtype) -> dict:
        """The four filters as tensors; ``rec_*_rev`` are time-reversed (``wavelets.py:81-90``)."""
        return _as_tensors(self, torch.device(device), dtype)


WaveletLike = Union[str, FilterBank, Sequence[Sequence[float]], "pywt.Wavelet"]  # noqa: F821

_CONTINUOUS = ("morl", "morlet", "cmor", "mexh", "gaus1", "shan", "fbsp")


def _as_floats(f: Sequence[float]) -> tuple:
    return tuple(float(v) for v in f)


def get_filter_bank(wavelet: WaveletLike) -> FilterBank:
    """A :class:`FilterBank` from a name (``"haar"``, ``"db4"``, ..., any PyWavelets name when
    PyWavelets is installed), a ``pywt.Wavelet``-like object (``.filter_bank``, ``.name``), a
    :class:`FilterBank`, or four sequences ``(dec_lo, dec_hi, rec_lo, rec_hi)``
    (``wavelets.py:44-64``).  The four filters are zero-padded at the end to the longest one's
    length, rounded up to even; trailing zeros leave the transform unchanged.
    """
    if isinstance(wavelet, FilterBank):
        return wavelet
    if isinstance(wavelet, str):
        return _named_bank(wavelet)
    source = getattr(wavelet, "filter_bank", None)
    name = getattr(wavelet, "name", "custom") if source is not None else "custom"
    filters = source if source is not None else wavelet
    if len(filters) != 4:
        raise ValueError("a custom filter bank must be (dec_lo, dec_hi, rec_lo, rec_hi)")
    filters = [_as_floats(f) for f in filters]
    even = -(-max(len(f) for f in filters) // 2) * 2
    return FilterBank(name, *(f + (0.0,) * (even - len(f)) for f in filters))


def daubechies_scaling_filter(order: int) -> np.ndarray:
    """Minimum-phase Daubechies scaling filter with ``order`` vanishing moments (2*order taps).

    Spectral factorisation (Daubechies 1988): ``|m0|^2 = cos^{2N}(w/2) P(sin^2(w/2))`` with
    ``P(y) = sum_{k<N} C(N-1+k, k) y^k``.  Each root ``y_i`` of ``P`` gives a pair of
    reciprocal roots of ``z^2 - (2 - 4 y_i) z + 1``; the one inside the unit circle is kept.
    The filter is the real polynomial ``(1+z)^N prod (z - z_i)`` normalised to ``sum h = sqrt 2``.
    """
    if order < 1:
        raise ValueError("the Daubechies order must be >= 1")
    p = [comb(order - 1 + k, k) for k in range(order)]
    y_roots = np.roots(p[::-1]) if order > 1 else np.zeros(0)
    poly = np.array([1.0 + 0j])
    for _ in range(order):
        poly = np.convolve(poly, [1.0, 1.0])
    for y in y_roots:
        b = 1.0 - 2.0 * y
        s = np.sqrt(b * b - 1.0 + 0j)
        z = b + s if abs(b + s) < 1.0 else b - s
        poly = np.convolve(poly, [1.0, -z])
    h = np.real(poly)
    return h * (np.sqrt(2.0) / h.sum())


def _orthogonal_bank(name: str, h: np.ndarray) -> FilterBank:
    L = len(h)
    rec_lo = [float(v) for v in h]
    rec_hi = [float((-1) ** k * h[L - 1 - k]) for k in range(L)]
    return FilterBank(name, tuple(rec_lo[::-1]), tuple(rec_hi[::-1]), tuple(rec_lo), tuple(rec_hi))


@lru_cache(maxsize=None)
def _named_bank(name: str) -> FilterBank:
    if name.lower() in _CONTINUOUS:
        raise ValueError(
            f"'{name}' is a continuous wavelet without a finite two-channel filter bank; "
            "use cwt / CWT1D for the Morlet transform."
        )
    try:
        import pywt  # noqa: F401
    except ImportError:
        pywt = None
    if pywt is not None:
        return get_filter_bank(pywt.Wavelet(name))
    m = re.fullmatch(r"db(\d+)", name)
    if name == "haar" or (m and int(m.group(1)) >= 1):
        order = 1 if name == "haar" else int(m.group(1))
        if order > 20:
            raise ImportError(f"PyWavelets is required for '{name}' (orders above 20)")
        return _orthogonal_bank(name, daubechies_scaling_filter(order))
    raise ImportError(f"PyWavelets is required to look up the wavelet '{name}' by name")


@lru_cache(maxsize=None)
def _as_tensors(bank: FilterBank, device: torch.device, dtype: torch.dtype) -> dict:
    """The analysis filters as they are, the synthesis filters time-reversed (the reference's
    synthesis is the transpose of an analysis by the reversed filters)."""
    taps = {"dec_lo": bank.dec_lo, "dec_hi": bank.dec_hi,
            "rec_lo_rev": bank.rec_lo[::-1], "rec_hi_rev": bank.rec_hi[::-1]}
    return {k: torch.tensor(v, dtype=dtype, device=device) for k, v in taps.items()}
