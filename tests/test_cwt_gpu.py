"""Morlet CWT, fused mix and spectral softmax on the GPU: sm_100a kernels (through the C ABI)
vs the golden fixtures of the reference's CPU path and the CPU oracle.

Tolerances: fp64 1e-10 x max|ref| (the reference's own GPU-vs-CPU bound,
tests/test_cwt.py:192), fp32 1e-4 relative to max|ref| (the north-star bound for CWT, mixer
and softmax outputs and gradients).
"""

import math

import numpy as np
import pytest
import torch

import pytorch_morlet_fdwt_b200 as F
from pytorch_morlet_fdwt_b200.cwt import _apply_plan, morlet_mix, spectral_softmax
from oracle import cwt_oracle as C
from tests.golden_data import golden

pytestmark = pytest.mark.gpu
DEV = "cuda"
FREQS = np.geomspace(0.5, 100, 24)


def close(a, b, tol):
    a = a.detach().cpu() if torch.is_tensor(a) else torch.as_tensor(a)
    b = b.detach().cpu() if torch.is_tensor(b) else torch.as_tensor(b)
    if a.is_complex():
        a = torch.view_as_real(a)
    if b.is_complex():
        b = torch.view_as_real(b)
    a, b = a.double(), b.double()
    assert a.shape == b.shape, (a.shape, b.shape)
    scale = float(b.abs().max()) if b.numel() else 1.0
    err = float((a - b).abs().max()) if b.numel() else 0.0
    assert err <= tol * max(scale, 1e-300), f"max err {err:.3e} > {tol:.1e} x {scale:.3e}"


@pytest.mark.parametrize("case", [("fast", "l1", True, 4.0), ("fast", "l2", False, 4.0),
                                  ("direct", "l2", True, 4.0), ("fast", "l2", True, 5.0)])
def test_cwt_vs_golden(case):
    g = golden("cwt")
    method, norm, cplx, trunc = case
    x = torch.from_numpy(g["cwt|x"]).to(DEV)
    y = F.cwt(x, freqs=np.geomspace(1, 60, 8), fs=250.0, method=method, norm=norm,
              complex=cplx, truncate=trunc)
    y = torch.view_as_real(y) if cplx else y
    close(y, g[f"cwt|{method}|{norm}|{int(cplx)}|{trunc:g}"], 1e-10)


def _naive_cwt(x, scales, w0=6.0, truncate=4.0):
    """Literal definition W[s, n] = sum_m x[m] conj(psi((m - n)/s)) / sqrt(s)."""
    N = x.shape[-1]
    m = torch.arange(N, dtype=torch.float64)
    out = []
    for s in scales:
        t = (m[None, :] - m[:, None]) / s
        env = torch.exp(-0.5 * t ** 2) * ((m[None, :] - m[:, None]).abs() <= math.ceil(truncate * s))
        psi = math.pi ** -0.25 * (torch.exp(1j * w0 * t) - math.exp(-w0 ** 2 / 2)) * env
        out.append((x.to(torch.complex128) @ psi.conj().T) / math.sqrt(s))
    return torch.stack(out, -2)


def test_direct_and_fft_match_definition():
    torch.manual_seed(0)
    x = torch.randn(2, 300, dtype=torch.float64)
    scales = [1.0, 2.5, 7.0, 30.0]
    ref = _naive_cwt(x, scales)
    for method in ["direct", "fft"]:
        out = F.cwt(x.to(DEV), scales, method=method).cpu()
        torch.testing.assert_close(out, ref, atol=1e-12, rtol=0)


@pytest.mark.parametrize("n", [7, 500, 3000])
def test_methods_agree(n):
    torch.manual_seed(0)
    x = torch.randn(3, n, dtype=torch.float64, device=DEV)
    ref = F.cwt(x, freqs=FREQS, fs=250, method="direct")
    scale = ref.abs().max()
    torch.testing.assert_close(F.cwt(x, freqs=FREQS, fs=250, method="fft"), ref,
                               atol=1e-12 * scale, rtol=0)
    fast = F.cwt(x, freqs=FREQS, fs=250, method="fast")
    assert ((fast - ref).abs().max() / scale) < 3e-4
    torch.testing.assert_close(fast[..., -4:, :], ref[..., -4:, :], atol=1e-12 * scale, rtol=0)


def test_cfg3_forward_fp32_vs_oracle():
    """40 freqs logspace(-0.3, 2) at 250 Hz, l1, fast, on (32, 64, 2500) fp32;
    sampled rows against the oracle (fp64), every row finite."""
    torch.manual_seed(3)
    freqs = np.logspace(-0.3, 2, 40)
    x = torch.randn(32, 64, 2500, device=DEV)
    y = F.cwt(x, freqs=freqs, fs=250.0, norm="l1")
    assert y.shape == (32, 64, 40, 2500) and y.dtype == torch.complex64
    assert torch.isfinite(torch.view_as_real(y)).all()
    rows = [0, 5, 1000, 2047]
    p = C.Plan(C.freqs_to_scales(freqs, 250.0), norm="l1")
    H = p.filters(torch.tensor(p.scales, dtype=torch.float64), p.w0)
    xr = x.reshape(-1, 2500)[rows].double().cpu()
    ref = C.apply_plan(xr, p, H)
    close(y.reshape(-1, 40, 2500)[rows], ref, 1e-4)


def test_fp32_accuracy_and_dtypes():
    torch.manual_seed(0)
    x = torch.randn(8, 2500, device=DEV)
    ref = F.cwt(x.double(), freqs=FREQS, fs=250, method="fast")
    out = F.cwt(x, freqs=FREQS, fs=250, method="fast")
    assert out.dtype == torch.complex64
    assert ((out - ref).abs().max() / ref.abs().max()) < 1e-5
    out16 = F.cwt(x.half(), freqs=FREQS, fs=250, method="fast")
    assert out16.dtype == torch.complex64
    assert ((out16 - ref).abs().max() / ref.abs().max()) < 1e-2


def test_frequency_localisation():
    fs, f0 = 250.0, 10.0
    t = torch.arange(5000, dtype=torch.float64, device=DEV) / fs
    x = torch.sin(2 * math.pi * f0 * t)
    freqs = np.geomspace(1, 60, 40)
    for norm in ["l1", "l2"]:
        w = F.cwt(x, freqs=freqs, fs=fs, norm=norm).abs()[:, 2000:3000].mean(-1)
        assert abs(freqs[int(w.argmax())] - f0) / f0 < 0.06
    amps = []
    for f in [3.0, 12.0, 40.0]:
        x = torch.sin(2 * math.pi * f * t)
        amps.append(float(F.cwt(x, freqs=[f], fs=fs, norm="l1").abs()[0, 2000:3000].mean()))
    assert max(amps) / min(amps) < 1.01


def test_filters_are_exactly_symmetric_on_device():
    """The fused kernels take the one-FMA-per-tap-pair path only for exactly even/odd filters;
    MorletPlan.filters on the GPU must produce them."""
    m = F.CWT1D(freqs=np.logspace(-0.3, 2, 40), fs=250, learnable=True, learnable_w0=True)
    H = m.plan.filters(m.log_scales.to(torch.float64).exp().cuda(), torch.tensor(6.3).cuda(),
                       torch.float32)
    c = m.plan.center
    Hr, Hi = H[0::2], H[1::2]
    k = torch.arange(1, c + 1, device=DEV)
    assert torch.equal(Hr[:, c + k], Hr[:, c - k])
    assert torch.equal(Hi[:, c + k], -Hi[:, c - k])


def test_mix_forward_vs_oracle():
    torch.manual_seed(0)
    for cplx in (True, False):
        plan_m = F.CWT1D(freqs=np.geomspace(1, 60, 12), fs=250, complex=cplx, learnable=True)
        B, D, N = 2, 3, 1500
        x = torch.randn(B, D, N, dtype=torch.float64)
        a = torch.randn(D, 12, dtype=torch.float64)
        b = torch.randn(D, 12, dtype=torch.float64)
        p = plan_m.plan
        H = p.filters(plan_m.log_scales.to(torch.float64).exp(), p.w0, torch.float64)
        y = morlet_mix(x.to(DEV), p, H.to(DEV), a.to(DEV), b.to(DEV))
        po = C.Plan(p.scales, complex=cplx, support_margin=1.25)
        ref = C.mix(x, po, H, a, b)
        close(y, ref, 1e-10)


@pytest.mark.parametrize("per_position", [False, True])
def test_spectral_softmax_forward_vs_oracle(per_position):
    torch.manual_seed(0)
    m = F.CWT1D(scales=[1.5, 3.0, 7.0, 13.0, 26.0], learnable=True, learnable_w0=True).double()
    nch, R, N = 3, 6, 80
    x = torch.randn(R, N, dtype=torch.float64)
    shape = (R // nch, 5, N) if per_position else (nch, 5)
    V = torch.randn(shape, dtype=torch.float64)
    H = m.plan.filters(m.log_scales.exp(), m.w0, torch.float64)
    out = spectral_softmax(x.to(DEV), m.plan, H.to(DEV), V.to(DEV), nch, 0.7)
    po = C.Plan(m.plan.scales, support_margin=1.25)
    ref = C.spectral_softmax(x, po, H.detach(), V, nch, 0.7)
    close(out, ref, 1e-10)


def test_layers_forward_vs_golden():
    g = golden("layers")
    P = {n.split("|", 2)[2]: torch.from_numpy(g[n]) for n in g.files if n.startswith("mixer|p|")}
    mixer = F.MorletTokenMixer(8, freqs=np.geomspace(1, 40, 6).tolist(), fs=250).double()
    mixer.load_state_dict({k: v for k, v in P.items()}, strict=False)
    with torch.no_grad():
        for k, v in P.items():
            dict(mixer.named_parameters())[k].copy_(v)
    mixer = mixer.to(DEV)
    y = mixer(torch.from_numpy(g["mixer|x"]).to(DEV))
    close(y, g["mixer|y"], 1e-10)
    for cls, key in [(F.MorletAttention, "MorletAttention"),
                     (F.MorletChannelMixAttention, "MorletChannelMixAttention")]:
        m = cls(num_channels=3, hidden_dim=64, temperature=0.5).double()
        with torch.no_grad():
            for name, prm in m.named_parameters():
                prm.copy_(torch.from_numpy(g[f"{key}|p|{name}"]))
        m = m.to(DEV)
        y = m(torch.from_numpy(g[key + "|x"]).to(DEV))
        close(y, g[key + "|y"], 1e-10)
    # large amplitudes and a small temperature: the online softmax stays finite
    m = F.MorletAttention(num_channels=2, hidden_dim=100, temperature=0.01).double()
    with torch.no_grad():
        for name, prm in m.named_parameters():
            prm.copy_(torch.from_numpy(g[f"attn_large|p|{name}"]))
    y = m.to(DEV)(torch.from_numpy(g["attn_large|x"]).to(DEV))
    assert torch.isfinite(y).all()
    close(y, g["attn_large|y"], 1e-10)
