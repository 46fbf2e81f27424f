"""Backward passes of the Morlet CWT, the fused mix and the spectral softmax on the GPU
(sm_100a kernels through the C ABI) against the golden gradients of the reference's CPU path
and the autograd gradients of the CPU oracle.

Tolerances: fp64 1e-10 x max|ref| (the reference's own GPU-vs-CPU bound for gradients,
tests/test_cwt.py:75-77), fp32 1e-4 relative to max|ref| (the north-star bound for gradients).
"""

import numpy as np
import pytest
import torch
from torch.autograd import gradcheck, gradgradcheck

import pytorch_morlet_fdwt_b200 as F
from pytorch_morlet_fdwt_b200.cwt import _apply_plan, morlet_mix, spectral_softmax
from oracle import cwt_oracle as C
from tests.golden_data import golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def close(a, b, tol):
    a = a.detach().cpu() if torch.is_tensor(a) else torch.as_tensor(a)
    b = b.detach().cpu() if torch.is_tensor(b) else torch.as_tensor(b)
    a, b = a.double(), b.double()
    assert a.shape == b.shape, (a.shape, b.shape)
    scale = float(b.abs().max()) if b.numel() else 1.0
    err = float((a - b).abs().max()) if b.numel() else 0.0
    assert err <= tol * max(scale, 1e-300), f"max err {err:.3e} > {tol:.1e} x {scale:.3e}"


@pytest.mark.parametrize("cplx", [True, False])
def test_learnable_cwt_grads_vs_golden(cplx):
    g = golden("cwt")
    key = f"cwtlearn|{int(cplx)}"
    m = F.CWT1D(freqs=np.geomspace(1, 60, 8)[:6], fs=250.0, learnable=True, learnable_w0=True,
                complex=cplx).double().to(DEV)
    x = torch.from_numpy(g[key + "|x"]).to(DEV).requires_grad_()
    y = m(x)
    (y.abs().square().sum() if cplx else (y.square() * 1.5).sum()).backward()
    close(x.grad, g[key + "|gx"], 1e-10)
    close(m.log_scales.grad, g[key + "|gls"], 1e-10)
    close(m.w0.grad, g[key + "|gw0"], 1e-10)


@pytest.mark.parametrize("method", ["direct", "fast"])
@pytest.mark.parametrize("cplx", [True, False])
def test_gradcheck(method, cplx):
    torch.manual_seed(0)
    scales = [1.5, 3.0, 6.0, 9.0, 14.0, 23.0]
    m = F.CWT1D(scales=scales, method=method, complex=cplx, learnable=True,
                learnable_w0=True).to(DEV).double()
    for n in [5, 37, 150]:
        x = torch.randn(2, n, dtype=torch.float64, device=DEV, requires_grad=True)
        ls = m.log_scales.detach().clone().requires_grad_()
        w0 = torch.tensor(6.0, dtype=torch.float64, device=DEV, requires_grad=True)

        def f(ls, w0, x):
            y = _apply_plan(x, m.plan, m.plan.filters(ls.exp(), w0, torch.float64))
            return torch.view_as_real(y) if cplx else y

        assert gradcheck(f, (ls, w0, x))


@pytest.mark.parametrize("cplx", [True, False])
def test_gradgradcheck(cplx):
    """Second derivatives: the backward node is itself built from the forward, adjoint and
    filter-gradient kernels."""
    torch.manual_seed(1)
    m = F.CWT1D(scales=[1.5, 4.0, 11.0, 23.0], complex=cplx, learnable=True,
                learnable_w0=True).to(DEV).double()
    x = torch.randn(2, 37, dtype=torch.float64, device=DEV, requires_grad=True)
    ls = m.log_scales.detach().clone().requires_grad_()
    w0 = torch.tensor(6.0, dtype=torch.float64, device=DEV, requires_grad=True)

    def f(ls, w0, x):
        y = _apply_plan(x, m.plan, m.plan.filters(ls.exp(), w0, torch.float64))
        return torch.view_as_real(y) if cplx else y

    assert gradgradcheck(f, (ls, w0, x))


def test_cfg3_learnable_backward_fp32_vs_oracle():
    """configs[2] with learnable scales and w0: loss sum |W|^2 on (32, 64, 2500) fp32; dL/dx on
    sampled rows and dL/dH over a row subset against the fp64 oracle."""
    torch.manual_seed(3)
    freqs = np.logspace(-0.3, 2, 40)
    m = F.CWT1D(freqs=freqs, fs=250.0, norm="l1", learnable=True, learnable_w0=True).to(DEV)
    x = torch.randn(32, 64, 2500, device=DEV, requires_grad=True)
    y = m(x)
    y.abs().square().sum().backward()
    assert torch.isfinite(x.grad).all() and torch.isfinite(m.log_scales.grad).all()
    rows = [0, 7, 1000, 2047]
    po = C.Plan(m.plan.scales, norm="l1", support_margin=1.25)
    ls = m.log_scales.detach().double().cpu().requires_grad_()
    w0 = m.w0.detach().double().cpu().requires_grad_()
    xr = x.detach().reshape(-1, 2500)[rows].double().cpu().requires_grad_()
    W = C.apply_plan(xr, po, po.filters(ls.exp(), w0))
    W.abs().square().sum().backward()
    close(x.grad.reshape(-1, 2500)[rows], xr.grad, 1e-4)
    # filter gradients over the same rows, from the GPU
    m.zero_grad()
    xs = x.detach().reshape(-1, 2500)[rows].clone().requires_grad_()
    m(xs).abs().square().sum().backward()
    close(m.log_scales.grad, ls.grad, 1e-4)
    close(m.w0.grad, w0.grad, 1e-4)


@pytest.mark.parametrize("cplx", [True, False])
def test_mix_backward_vs_oracle(cplx):
    torch.manual_seed(0)
    mod = F.CWT1D(freqs=np.geomspace(1, 60, 12), fs=250, complex=cplx, learnable=True,
                  learnable_w0=True).double()
    B, D, N = 2, 3, 700
    x = torch.randn(B, D, N, dtype=torch.float64)
    a = torch.randn(D, 12, dtype=torch.float64)
    b = torch.randn(D, 12, dtype=torch.float64)
    gy = torch.randn(B, D, N, dtype=torch.float64)
    p = mod.plan
    res = []
    for dev in ["gpu", "oracle"]:
        ls = mod.log_scales.detach().clone().requires_grad_()
        w0 = torch.tensor(6.0, dtype=torch.float64, requires_grad=True)
        xx, aa, bb = (t.clone().requires_grad_() for t in (x, a, b))
        if dev == "gpu":
            lsd, w0d = ls.to(DEV), w0.to(DEV)
            H = p.filters(lsd.exp(), w0d, torch.float64)
            y = morlet_mix(xx.to(DEV), p, H, aa.to(DEV), bb.to(DEV)).cpu()
        else:
            po = C.Plan(p.scales, complex=cplx, support_margin=1.25)
            y = C.mix(xx, po, po.filters(ls.exp(), w0), aa, bb)
        (y * gy).sum().backward()
        res.append([y, xx.grad, aa.grad, bb.grad, ls.grad, w0.grad])
    for u, v in zip(*res):
        close(u, v, 1e-10)


@pytest.mark.parametrize("per_position", [False, True])
def test_spectral_softmax_backward_vs_oracle(per_position):
    torch.manual_seed(0)
    m = F.CWT1D(scales=[1.5, 3.0, 7.0, 13.0, 26.0], learnable=True, learnable_w0=True).double()
    nch, R, N = 3, 6, 80
    x = torch.randn(R, N, dtype=torch.float64)
    shape = (R // nch, 5, N) if per_position else (nch, 5)
    V = torch.randn(shape, dtype=torch.float64)
    gy = torch.randn(R, N, dtype=torch.float64)
    res = []
    for dev in ["gpu", "oracle"]:
        ls = m.log_scales.detach().clone().requires_grad_()
        w0 = torch.tensor(6.0, dtype=torch.float64, requires_grad=True)
        xx, VV = x.clone().requires_grad_(), V.clone().requires_grad_()
        if dev == "gpu":
            H = m.plan.filters(ls.to(DEV).exp(), w0.to(DEV), torch.float64)
            out = spectral_softmax(xx.to(DEV), m.plan, H, VV.to(DEV), nch, 0.7).cpu()
        else:
            po = C.Plan(m.plan.scales, support_margin=1.25)
            out = C.spectral_softmax(xx, po, po.filters(ls.exp(), w0), VV, nch, 0.7)
        (out * gy).sum().backward()
        res.append([out, xx.grad, VV.grad, ls.grad, w0.grad])
    for u, v in zip(*res):
        close(u, v, 1e-10)


def test_layers_backward_vs_golden():
    g = golden("layers")
    P = {n.split("|", 2)[2]: torch.from_numpy(g[n]) for n in g.files if n.startswith("mixer|p|")}
    mixer = F.MorletTokenMixer(8, freqs=np.geomspace(1, 40, 6).tolist(), fs=250).double()
    with torch.no_grad():
        for k, v in P.items():
            dict(mixer.named_parameters())[k].copy_(v)
    mixer = mixer.to(DEV)
    x = torch.from_numpy(g["mixer|x"]).to(DEV).requires_grad_()
    mixer(x).square().sum().backward()
    close(x.grad, g["mixer|gx"], 1e-10)
    for name, prm in mixer.named_parameters():
        close(prm.grad, g[f"mixer|g|{name}"], 1e-10)
    for cls, key in [(F.MorletAttention, "MorletAttention"),
                     (F.MorletChannelMixAttention, "MorletChannelMixAttention")]:
        m = cls(num_channels=3, hidden_dim=64, temperature=0.5).double()
        with torch.no_grad():
            for name, prm in m.named_parameters():
                prm.copy_(torch.from_numpy(g[f"{key}|p|{name}"]))
        m = m.to(DEV)
        x = torch.from_numpy(g[key + "|x"]).to(DEV).requires_grad_()
        m(x).square().sum().backward()
        close(x.grad, g[key + "|gx"], 1e-10)
        for name, prm in m.named_parameters():
            close(prm.grad, g[f"{key}|g|{name}"], 1e-10)


def test_backward_without_filter_grad_and_fp32_dtypes():
    """x-only gradients (fixed filters) and fp32 against fp64."""
    torch.manual_seed(2)
    x = torch.randn(4, 1800, dtype=torch.float64, device=DEV)
    freqs = np.geomspace(0.5, 100, 24)
    g = torch.randn(4, 24, 1800, dtype=torch.complex128, device=DEV)
    outs = []
    for dt in (torch.float64, torch.float32):
        xx = x.detach().clone().to(dt).requires_grad_()
        y = F.cwt(xx, freqs=freqs, fs=250)
        (y * g.to(y.dtype)).real.sum().backward()
        outs.append(xx.grad)
    close(outs[1], outs[0], 1e-4)
