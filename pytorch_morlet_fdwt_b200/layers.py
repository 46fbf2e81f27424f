"""Token-mixing layers built on the wavelet transforms (``fdwt/layers.py`` of the reference).

``MorletTokenMixer`` and ``WaveletTokenMixer`` map ``(batch, length, dim)`` to the same shape;
``MorletAttention`` and ``MorletChannelMixAttention`` work on multi-channel patch tokens
``(B, H, C, T, D)``.  Parameters, initialisation and state-dict keys match the reference.
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


class MorletTokenMixer(nn.Module):
    """Mix tokens through a Morlet scalogram (``fdwt/layers.py:26-72``)::

        y[b, l, d] = sum_s mag_weight[d, s] |W_s x[b, :, d]|(l) + phase_weight[d, s] Re W_s x(l)

    then ``+ bias`` and the ``out_proj`` linear layer.  The scalogram is never materialised.
    """

    def __init__(self, dim: int, freqs: Optional[Sequence[float]] = None,
                 scales: Optional[Sequence[float]] = None, fs: float = 1.0, w0: float = 6.0,
                 method: str = "fast", learnable_scales: bool = True, use_phase: bool = True,
                 out_proj: bool = True):
        super().__init__()
        if freqs is None and scales is None:
            scales = torch.logspace(0, 6, 16, base=2).tolist()  # 1 .. 64 tokens
        self.cwt = CWT1D(freqs=freqs, scales=scales, fs=fs, w0=w0, method=method,
                         learnable=learnable_scales)
        S = self.cwt.plan.num_scales
        self.use_phase = use_phase
        self.mag_weight = nn.Parameter(torch.randn(dim, S) / S ** 0.5)
        self.phase_weight = nn.Parameter(torch.randn(dim, S) / S ** 0.5, requires_grad=use_phase)
        if not use_phase:
            self.phase_weight.data.zero_()
        self.bias = nn.Parameter(torch.zeros(dim))
        self.out_proj = nn.Linear(dim, dim) if out_proj else nn.Identity()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = torch.float64 if x.dtype == torch.float64 else torch.float32
        H = self.cwt._filters(x.device, dt)
        # the kernels read the (B, L, D) tokens and write y + bias in the same layout
        y = morlet_mix_tokens(x, self.cwt.plan, H, self.mag_weight, self.phase_weight, self.bias)
        return self.out_proj(y.to(x.dtype))


class WaveletTokenMixer(nn.Module):
    """Mix tokens in the DWT domain (``fdwt/layers.py:75-109``): fused multilevel DWT, a
    per-band channel MLP, fused multilevel inverse."""

    def __init__(self, dim: int, wavelet: WaveletLike = "db4", mode: str = "periodization",
                 level: int = 4, hidden: int = 0):
        super().__init__()
        if level < 1:
            raise ValueError("level must be >= 1")
        self.wavelet, self.mode, self.level = wavelet, mode, level

        def band():
            if hidden:
                return nn.Sequential(nn.Linear(dim, hidden), nn.GELU(), nn.Linear(hidden, dim))
            return nn.Linear(dim, dim)

        self.bands = nn.ModuleList(band() for _ in range(level + 1))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        L = x.shape[1]
        coeffs = wavedec(x.transpose(1, 2), self.wavelet, self.mode, self.level)  # (B, D, n_j)
        mixed = [band(c.transpose(1, 2)).transpose(1, 2) for band, c in zip(self.bands, coeffs)]
        y = waverec(mixed, self.wavelet, self.mode)[..., :L]
        return y.transpose(1, 2)


class _MorletPatchAttention(nn.Module):
    """Shared plumbing (``fdwt/layers.py:112-162``): (B, H, C, T, D) patch tokens flattened to
    (B, H, C, T*D) signals sampled at ``hidden_dim / patch_duration`` Hz, a learnable CWT."""

    def __init__(self, num_channels: int, hidden_dim: int, freqs: Optional[Sequence[float]],
                 patch_duration: float, w0: float, learnable: bool, temperature: float,
                 method: str):
        super().__init__()
        self.num_channels, self.hidden_dim = num_channels, hidden_dim
        fs = hidden_dim / patch_duration
        if freqs is None:
            f_max = min(40.0, fs / 4)
            freqs = torch.logspace(0, math.log10(max(f_max, 1.5)), 16).tolist()
        if max(freqs) >= fs / 2:
            raise ValueError(f"frequencies must be below the Nyquist frequency {fs / 2:g} Hz")
        self.cwt = CWT1D(freqs=freqs, fs=fs, w0=w0, method=method,
                         learnable=learnable, learnable_w0=learnable)
        self.temperature = temperature

    @property
    def num_freqs(self) -> int:
        return self.cwt.plan.num_scales

    @property
    def freqs(self) -> torch.Tensor:
        """Current (learned) centre frequencies in Hz."""
        return self.cwt.freqs

    def _check(self, x: torch.Tensor):
        if x.dim() != 5:
            raise ValueError(f"expected (B, H, C, T, D) input, got shape {tuple(x.shape)}")
        B, H, C, T, D = x.shape
        if C != self.num_channels or D != self.hidden_dim:
            raise ValueError(f"expected C={self.num_channels} and D={self.hidden_dim}, "
                             f"got C={C} and D={D}")
        return B, H, C, T, D

    def _probs(self, x: torch.Tensor) -> torch.Tensor:
        """softmax_f |W_f x| / tau, shape (B, H, C, f, T*D) -- materialised (inspection)."""
        B, H, C, T, D = self._check(x)
        w = self.cwt(x.reshape(B, H, C, T * D))
        return torch.softmax(w.abs() / self.temperature, dim=-2)

    def _spectral_softmax(self, x: torch.Tensor, V: torch.Tensor) -> torch.Tensor:
        """sum_f softmax_f(|W_f x| / tau) V_f -> (B, H, C, T, D), one fused kernel."""
        B, H, C, T, D = x.shape
        dt = torch.float64 if x.dtype == torch.float64 else torch.float32
        Hf = self.cwt._filters(x.device, dt)
        out = spectral_softmax(x.reshape(B * H * C, T * D), self.cwt.plan, Hf, V, C,
                               self.temperature)
        return out.reshape(B, H, C, T, D).to(x.dtype)


class MorletAttention(_MorletPatchAttention):
    """``out[c, n] = sum_f softmax_f(|W_f x_c|(n) / temperature) * w[c, f]`` with a learned
    (C, f) matrix ``freq_weight`` (``fdwt/layers.py:165-218``)."""

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
    """Channel attention through a learned (f, C) frequency-to-channel map ``M``
    (``fdwt/layers.py:221-262``): ``out[c, n] = sum_f P[c, n, f] U[f, n]``, ``U = M x``."""

    def __init__(self, num_channels: int, hidden_dim: int,
                 freqs: Optional[Sequence[float]] = None, patch_duration: float = 1.0,
                 w0: float = 6.0, learnable: bool = True, temperature: float = 1.0,
                 method: str = "fast"):
        super().__init__(num_channels, hidden_dim, freqs, patch_duration, w0, learnable,
                         temperature, method)
        self.freq_to_channel = nn.Parameter(torch.randn(self.num_freqs, num_channels)
                                            / self.num_freqs ** 0.5)

    def attention_map(self, x: torch.Tensor) -> torch.Tensor:
        """Explicit (B, H, T*D, C, C) attention map, for inspection (memory heavy)."""
        p = self._probs(x)
        return torch.einsum("bhcfn,fk->bhnck", p, self.freq_to_channel.to(p.dtype))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, H, C, T, D = self._check(x)
        dt = torch.float64 if x.dtype == torch.float64 else torch.float32
        v = x.reshape(B, H, C, T * D).to(dt)
        U = torch.einsum("fk,bhkn->bhfn", self.freq_to_channel.to(dt), v)
        return self._spectral_softmax(x, U.reshape(B * H, self.num_freqs, T * D))
