"""Second derivatives through the fused scalogram consumers (the mix behind MorletTokenMixer,
the spectral softmax behind MorletAttention and MorletChannelMixAttention) on the GPU.

With create_graph=True their backward recomputes the consumer through the transform node, whose
derivatives of every order come from the sm_100a kernels; the results are compared with
``gradgradcheck`` and with the fp64 CPU oracle's autograd (the reference's CPU path is
twice-differentiable the same way, ``fdwt/cwt.py:391-394, 545-549``).

Tolerance: 1e-10 x max|ref| in fp64.
"""

import numpy as np
import pytest
import torch
from torch.autograd import gradgradcheck

import pytorch_morlet_fdwt_b200 as F
from pytorch_morlet_fdwt_b200.cwt import morlet_mix, spectral_softmax
from oracle import cwt_oracle as C

pytestmark = pytest.mark.gpu
DEV = "cuda"


def close(a, b, tol=1e-10, what=""):
    a = a.detach().cpu().double()
    b = b.detach().cpu().double()
    assert a.shape == b.shape, (what, a.shape, b.shape)
    scale = float(b.abs().max())
    err = float((a - b).abs().max())
    assert err <= tol * max(scale, 1e-300), f"{what}: max err {err:.3e} > {tol:.1e} x {scale:.3e}"


def test_gradgradcheck_mix():
    torch.manual_seed(0)
    m = F.CWT1D(scales=[1.5, 4.0, 11.0], learnable=True, learnable_w0=True).to(DEV).double()
    x = torch.randn(1, 2, 40, dtype=torch.float64, device=DEV, requires_grad=True)
    a = torch.randn(2, 3, dtype=torch.float64, device=DEV, requires_grad=True)
    b = torch.randn(2, 3, dtype=torch.float64, device=DEV, requires_grad=True)
    ls = m.log_scales.detach().clone().requires_grad_()

    def f(x, a, b, ls):
        return morlet_mix(x, m.plan, m.plan.filters(ls.exp(), 6.0, torch.float64), a, b)

    assert gradgradcheck(f, (x, a, b, ls))


@pytest.mark.parametrize("per_position", [False, True])
def test_gradgradcheck_spectral_softmax(per_position):
    torch.manual_seed(1)
    m = F.CWT1D(scales=[1.5, 4.0, 11.0], learnable=True, learnable_w0=True).to(DEV).double()
    nch, R, N = 2, 4, 30
    x = torch.randn(R, N, dtype=torch.float64, device=DEV, requires_grad=True)
    shape = (R // nch, 3, N) if per_position else (nch, 3)
    V = torch.randn(shape, dtype=torch.float64, device=DEV, requires_grad=True)
    w0 = torch.tensor(6.0, dtype=torch.float64, device=DEV, requires_grad=True)

    def f(x, V, w0):
        H = m.plan.filters(m.log_scales.detach().exp(), w0, torch.float64)
        return spectral_softmax(x, m.plan, H, V, nch, 0.7)

    assert gradgradcheck(f, (x, V, w0))


def _double_backward(model, x):
    """dL2/d(x, params) with L2 = |dL/dx|^2 and L = sum(y^2): a double backward."""
    y = model(x)
    (gx,) = torch.autograd.grad(y.square().sum(), x, create_graph=True)
    gx.square().sum().backward()
    return gx


def test_layers_double_backward_vs_oracle():
    torch.manual_seed(2)
    freqs = np.geomspace(1, 40, 5).tolist()
    mixer = F.MorletTokenMixer(6, freqs=freqs, fs=250).double()
    x = torch.randn(2, 200, 6, dtype=torch.float64)
    P = {k: v.detach().clone().requires_grad_() for k, v in mixer.named_parameters()}
    po = C.Plan(mixer.cwt.plan.scales, support_margin=1.25)

    def oracle_mixer(xx):
        H = po.filters(P["cwt.log_scales"].double().exp(), 6.0)
        return C.token_mixer(xx, po, H, P["mag_weight"], P["phase_weight"], P["bias"],
                             P["out_proj.weight"], P["out_proj.bias"])

    xo = x.clone().requires_grad_()
    go = _double_backward(oracle_mixer, xo)
    mixer = mixer.to(DEV)
    xg = x.to(DEV).requires_grad_()
    gg = _double_backward(mixer, xg)
    close(gg, go, what="mixer dL/dx")
    close(xg.grad, xo.grad, what="mixer d2")
    for k, prm in mixer.named_parameters():
        close(prm.grad, P[k].grad, what=f"mixer d2/{k}")

    for cls in (F.MorletAttention, F.MorletChannelMixAttention):
        torch.manual_seed(3)
        m = cls(num_channels=3, hidden_dim=40, temperature=0.6).double()
        x = torch.randn(1, 2, 3, 4, 40, dtype=torch.float64)
        P = {k: v.detach().clone().requires_grad_() for k, v in m.named_parameters()}
        po = C.Plan(m.cwt.plan.scales, support_margin=1.25)

        def oracle_att(xx, P=P, po=po, cls=cls):
            H = po.filters(P["cwt.log_scales"].double().exp(), P["cwt.w0"])
            if cls is F.MorletAttention:
                return C.attention(xx, po, H, P["freq_weight"], 0.6)
            return C.channel_mix_attention(xx, po, H, P["freq_to_channel"], 0.6)

        xo = x.clone().requires_grad_()
        go = _double_backward(oracle_att, xo)
        m = m.to(DEV)
        xg = x.to(DEV).requires_grad_()
        gg = _double_backward(m, xg)
        name = cls.__name__
        close(gg, go, what=f"{name} dL/dx")
        close(xg.grad, xo.grad, what=f"{name} d2")
        for k, prm in m.named_parameters():
            close(prm.grad, P[k].grad, what=f"{name} d2/{k}")
