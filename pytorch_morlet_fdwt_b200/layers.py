"""Token-mixing layers on the wavelet transforms, drop-ins for the reference's
``fdwt/layers.py``: the same classes, constructor arguments, parameter names and shapes, and
the same order of random initialisation (a model built after ``torch.manual_seed`` gets the
reference's parameters).  The forward passes run on this package's fused kernels.

- :class:`MorletTokenMixer`, ``(B, L, D) -> (B, L, D)``: every channel's Morlet scalogram,
  reduced over the scales by learned magnitude and real-part weights inside the kernel, which
  reads and writes the token layout itself (bias included); then ``out_proj``.
- :class:`WaveletTokenMixer`, ``(B, L, D) -> (B, L, D)``: multilevel DWT along L, one channel
  MLP per sub-band, inverse DWT.
- :class:`MorletAttention` and :class:`MorletChannelMixAttention`, ``(B, H, C, T, D)`` -> the
  same shape: each channel's T*D samples as one signal; per position, a softmax over the CWT
  frequencies weights learned per-channel values (or the channel-mixed input).
"""

from __future__ import annotations

import math
from typing import Optional, Sequence

import torch
from torch import nn

from .cwt import CWT1D, morlet_mix_tokens, spectral_softmax
from .dwt import wavedec, waverec
from .wavelets import WaveletLike

__all__ = ["MorletTokenMixer", "WaveletTokenMixer", "MorletAttention", "MorletChannelMixAttention"]


def _randn_over(rows: int, cols: int, fan: int) -> torch.Tensor:
    """Standard normal ``(rows, cols)`` weights scaled by ``1 / sqrt(fan)``."""
    return torch.randn(rows, cols) / fan ** 0.5


def _compute_dtype(x: torch.Tensor) -> torch.dtype:
    return torch.float64 if x.dtype == torch.float64 else torch.float32


class MorletTokenMixer(nn.Module):
    """Token mixing through a Morlet scalogram, linear in the sequence length
    (``fdwt/layers.py:26-72``)::

        y[b, l, d] = sum_s mag_weight[d, s] |W_s x[b, :, d]|(l) + phase_weight[d, s] Re W_s(l)

    plus ``bias[d]``, then ``out_proj`` (an ``nn.Linear``, or the identity).  Without
    ``freqs`` / ``scales`` the 16 scales are log-spaced from 1 to 64 tokens.  With
    ``use_phase=False`` the real-part weights are zero and frozen.  The scalogram is never
    stored: the kernels reduce it over the scales as they compute it.
    """

    def __init__(self, dim: int, freqs: Optional[Sequence[float]] = None,
                 scales: Optional[Sequence[float]] = None, fs: float = 1.0, w0: float = 6.0,
                 method: str = "fast", learnable_scales: bool = True, use_phase: bool = True,
                 out_proj: bool = True):
        super().__init__()
        if freqs is None and scales is None:
            scales = torch.logspace(0, 6, 16, base=2).tolist()
        self.cwt = CWT1D(freqs=freqs, scales=scales, fs=fs, w0=w0, method=method,
                         learnable=learnable_scales)
        n_scales = self.cwt.plan.num_scales
        self.use_phase = use_phase
        self.mag_weight = nn.Parameter(_randn_over(dim, n_scales, n_scales))
        phase = _randn_over(dim, n_scales, n_scales)  # drawn either way: keeps the RNG order
        if not use_phase:
            phase.zero_()
        self.phase_weight = nn.Parameter(phase, requires_grad=use_phase)
        self.bias = nn.Parameter(torch.zeros(dim))
        self.out_proj = nn.Linear(dim, dim) if out_proj else nn.Identity()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        filters = self.cwt._filters(x.device, _compute_dtype(x))
        mixed = morlet_mix_tokens(x, self.cwt.plan, filters, self.mag_weight, self.phase_weight,
                                  self.bias)
        return self.out_proj(mixed.to(x.dtype))


class WaveletTokenMixer(nn.Module):
    """Token mixing in the DWT domain (``fdwt/layers.py:75-109``): ``level`` levels of the
    multilevel DWT along the sequence, one channel map per sub-band (an ``nn.Linear``, or a
    ``Linear - GELU - Linear`` MLP of width ``hidden``), then the inverse DWT, trimmed to the
    input length."""

    def __init__(self, dim: int, wavelet: WaveletLike = "db4", mode: str = "periodization",
                 level: int = 4, hidden: int = 0):
        super().__init__()
        if level < 1:
            raise ValueError("level must be >= 1")
        self.wavelet = wavelet
        self.mode = mode
        self.level = level
        self.bands = nn.ModuleList([self._channel_map(dim, hidden) for _ in range(level + 1)])

    @staticmethod
    def _channel_map(dim: int, hidden: int) -> nn.Module:
        if not hidden:
            return nn.Linear(dim, dim)
        return nn.Sequential(nn.Linear(dim, hidden), nn.GELU(), nn.Linear(hidden, dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        n_tokens = x.shape[1]
        sub_bands = wavedec(x.transpose(1, 2), self.wavelet, self.mode, self.level)  # (B, D, n_j)
        mixed = [fn(c.transpose(1, 2)).transpose(1, 2) for fn, c in zip(self.bands, sub_bands)]
        y = waverec(mixed, self.wavelet, self.mode)
        return y[..., :n_tokens].transpose(1, 2)


def _default_freqs(fs: float) -> list:
    """16 centre frequencies log-spaced from 1 Hz to min(40 Hz, fs / 4), the top at least 1.5."""
    top = max(min(40.0, fs / 4), 1.5)
    return torch.logspace(0, math.log10(top), 16).tolist()


class _MorletPatchAttention(nn.Module):
    """What the two attention layers share (``fdwt/layers.py:112-162``): patch tokens
    ``(B, H, C, T, D)`` read as B*H*C signals of T*D samples at ``hidden_dim /
    patch_duration`` Hz, a learnable Morlet CWT of them, and the fused spectral softmax."""

    def __init__(self, num_channels: int, hidden_dim: int, freqs: Optional[Sequence[float]],
                 patch_duration: float, w0: float, learnable: bool, temperature: float,
                 method: str):
        super().__init__()
        self.num_channels = num_channels
        self.hidden_dim = hidden_dim
        fs = hidden_dim / patch_duration
        freqs = _default_freqs(fs) if freqs is None else freqs
        nyquist = fs / 2
        if max(freqs) >= nyquist:
            raise ValueError(f"frequencies must be below the Nyquist frequency {nyquist:g} Hz")
        self.cwt = CWT1D(freqs=freqs, fs=fs, w0=w0, method=method, learnable=learnable,
                         learnable_w0=learnable)
        self.temperature = temperature

    @property
    def num_freqs(self) -> int:
        return self.cwt.plan.num_scales

    @property
    def freqs(self) -> torch.Tensor:
        """The CWT's current centre frequencies in Hz."""
        return self.cwt.freqs

    def _check(self, x: torch.Tensor):
        """The input's ``(B, H, C, T, D)``, after checking its rank, C and D."""
        if x.dim() != 5:
            raise ValueError(f"expected (B, H, C, T, D) input, got shape {tuple(x.shape)}")
        dims = tuple(x.shape)
        if dims[2] != self.num_channels or dims[4] != self.hidden_dim:
            raise ValueError(f"expected C={self.num_channels} and D={self.hidden_dim}, "
                             f"got C={dims[2]} and D={dims[4]}")
        return dims

    def _probs(self, x: torch.Tensor) -> torch.Tensor:
        """The softmax over frequencies of ``|W x| / temperature``, materialised as
        ``(B, H, C, f, T*D)`` (for inspection; the layers themselves never store it)."""
        B, H, C, T, D = self._check(x)
        magnitude = self.cwt(x.reshape(B, H, C, T * D)).abs()
        return torch.softmax(magnitude / self.temperature, dim=-2)

    def _spectral_softmax(self, x: torch.Tensor, V: torch.Tensor) -> torch.Tensor:
        """``sum_f softmax_f(|W_f x| / temperature) V_f`` shaped like ``x``, in one fused
        kernel (V per channel ``(C, f)``, or per position ``(B*H, f, T*D)``)."""
        B, H, C, T, D = x.shape
        signals = x.reshape(B * H * C, T * D)
        filters = self.cwt._filters(x.device, _compute_dtype(x))
        out = spectral_softmax(signals, self.cwt.plan, filters, V, C, self.temperature)
        return out.reshape(B, H, C, T, D).to(x.dtype)


class MorletAttention(_MorletPatchAttention):
    """Attention whose query-key step is a Morlet spectrum (``fdwt/layers.py:165-218``).

    Channel c's T*D samples are one signal ``x_c``; at every position the layer returns a
    softmax-weighted average of the channel's learned per-frequency values::

        out[c, n] = sum_f softmax_f(|W_f x_c|(n) / temperature) * freq_weight[c, f]

    so the locally dominant frequencies decide which values count.  The CWT scales and wave
    number are learned too (``learnable``).  One fused kernel computes the CWT, the online
    softmax across its octaves and the weighting: only the output and two softmax statistics
    per position are stored, never the ``(B, H, C, f, T*D)`` scalogram.

    Args: ``num_channels`` (C), ``hidden_dim`` (D), ``freqs`` (Hz; 16 log-spaced from 1 Hz to
    ``min(40, fs / 4)`` by default), ``patch_duration`` (seconds per token, so that
    ``fs = hidden_dim / patch_duration``), ``w0``, ``learnable``, ``temperature``, ``method``.
    """

    def __init__(self, num_channels: int, hidden_dim: int,
                 freqs: Optional[Sequence[float]] = None, patch_duration: float = 1.0,
                 w0: float = 6.0, learnable: bool = True, temperature: float = 1.0,
                 method: str = "fast"):
        super().__init__(num_channels, hidden_dim, freqs, patch_duration, w0, learnable,
                         temperature, method)
        self.freq_weight = nn.Parameter(torch.randn(num_channels, self.num_freqs))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        self._check(x)
        return self._spectral_softmax(x, self.freq_weight)


class MorletChannelMixAttention(_MorletPatchAttention):
    """Channel attention driven by Morlet spectra (``fdwt/layers.py:221-262``).

    Each channel's softmaxed spectrum ``P[c, n, f]`` acts as its query; a learned ``(f, C)``
    matrix ``M = freq_to_channel`` maps it to weights over the channels, applied to the input
    itself::

        out[c, n] = sum_c' (sum_f P[c, n, f] M[f, c']) x_c'[n] = sum_f P[c, n, f] U[f, n],
        U[f, n] = sum_c' M[f, c'] x_c'[n].

    The C x C map is never formed (cost O(T*D C f)).  ``U`` is one small matmul; the CWT,
    softmax and weighting by ``U`` are the fused kernel of :class:`MorletAttention`.
    """

    def __init__(self, num_channels: int, hidden_dim: int,
                 freqs: Optional[Sequence[float]] = None, patch_duration: float = 1.0,
                 w0: float = 6.0, learnable: bool = True, temperature: float = 1.0,
                 method: str = "fast"):
        super().__init__(num_channels, hidden_dim, freqs, patch_duration, w0, learnable,
                         temperature, method)
        self.freq_to_channel = nn.Parameter(
            _randn_over(self.num_freqs, num_channels, self.num_freqs))

    def attention_map(self, x: torch.Tensor) -> torch.Tensor:
        """The explicit ``(B, H, T*D, C, C)`` channel-attention map (memory heavy; for
        inspection): ``A[n, c, c'] = sum_f P[c, n, f] M[f, c']``."""
        p = self._probs(x)                              # (B, H, C, f, N)
        m = self.freq_to_channel.to(p.dtype)            # (f, C')
        return torch.matmul(p.permute(0, 1, 4, 2, 3), m)  # (B, H, N, C, C')

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, H, C, T, D = self._check(x)
        values = x.reshape(B, H, C, T * D).to(_compute_dtype(x))
        U = torch.matmul(self.freq_to_channel.to(values.dtype), values)  # (B, H, f, T*D)
        return self._spectral_softmax(x, U.reshape(B * H, self.num_freqs, T * D))
