"""Morlet CWT, fused mix and spectral softmax on rows computed in time tiles (sm_100a kernels
through the C ABI), the path of rows too long for one CTA's shared memory.

* With the test hook fdwt_set_cwt_tile_test forcing short tiles, the tiled forward (tiles with
  the pyramid's halo) and the octave-tiled backward must reproduce the fp64 oracle, for every
  consumer, on rows where many tiles meet (and where tiles cover the margins past the row ends).
* Rows longer than one CTA's shared memory take the tiled path by themselves: the reference's
  README shapes (64 x 15000 CWT forward + backward, MorletTokenMixer at L = 16384), compared
  with the oracle on sampled rows.

Tolerances: fp64 1e-10 x max|ref|, fp32 1e-4 x max|ref|.
"""

import numpy as np
import pytest
import torch

import pytorch_morlet_fdwt_b200 as F
from pytorch_morlet_fdwt_b200 import _lib
from pytorch_morlet_fdwt_b200.cwt import morlet_mix, spectral_softmax
from oracle import cwt_oracle as C

pytestmark = pytest.mark.gpu
DEV = "cuda"


def close(a, b, tol, what=""):
    a = a.detach().cpu()
    b = b.detach().cpu()
    if a.is_complex():
        a = torch.view_as_real(a)
    if b.is_complex():
        b = torch.view_as_real(b)
    a, b = a.double(), b.double()
    assert a.shape == b.shape, (what, a.shape, b.shape)
    scale = float(b.abs().max())
    err = float((a - b).abs().max())
    assert err <= tol * max(scale, 1e-300), f"{what}: max err {err:.3e} > {tol:.1e} x {scale:.3e}"


@pytest.fixture
def tiles():
    def set_tiles(t):
        _lib.set_cwt_tile_test(t)
    yield set_tiles
    _lib.set_cwt_tile_test(0)


def _oracle_inputs(m):
    po = C.Plan(m.plan.scales, norm=m.plan.norm, complex=m.plan.complex,
                truncate=m.plan.truncate, support_margin=1.25 if m._learn else 1.0)
    ls = m.log_scales.detach().double().cpu().requires_grad_()
    w0 = m.w0.detach().double().cpu().requires_grad_()
    return po, ls, w0


@pytest.mark.parametrize("t_len", [256, 1024])
@pytest.mark.parametrize("cplx", [True, False])
def test_tiled_cwt_forward_backward_fp64(tiles, t_len, cplx):
    torch.manual_seed(4)
    m = F.CWT1D(freqs=np.geomspace(0.7, 90, 14), fs=250.0, norm="l1", complex=cplx,
                learnable=True, learnable_w0=True).to(DEV).double()
    x = torch.randn(3, 2100, dtype=torch.float64, device=DEV, requires_grad=True)
    tiles(t_len)
    y = m(x)
    g = torch.randn_like(torch.view_as_real(y) if cplx else y)
    ((torch.view_as_real(y) if cplx else y) * g).sum().backward()
    tiles(0)
    po, ls, w0 = _oracle_inputs(m)
    xo = x.detach().cpu().requires_grad_()
    yo = C.apply_plan(xo, po, po.filters(ls.exp(), w0))
    ((torch.view_as_real(yo) if cplx else yo) * g.cpu()).sum().backward()
    close(y, yo, 1e-10, "W")
    close(x.grad, xo.grad, 1e-10, "dL/dx")
    close(m.log_scales.grad, ls.grad, 1e-10, "dL/dlog_scales")
    close(m.w0.grad, w0.grad, 1e-10, "dL/dw0")


@pytest.mark.parametrize("t_len", [256, 768])
def test_tiled_mix_fp64(tiles, t_len):
    torch.manual_seed(5)
    m = F.CWT1D(freqs=np.geomspace(1, 60, 9), fs=250.0, learnable=True,
                learnable_w0=True).to(DEV).double()
    B, D, N = 2, 3, 1800
    x = torch.randn(B, D, N, dtype=torch.float64, device=DEV, requires_grad=True)
    a = torch.randn(D, 9, dtype=torch.float64, device=DEV, requires_grad=True)
    b = torch.randn(D, 9, dtype=torch.float64, device=DEV, requires_grad=True)
    gy = torch.randn(B, D, N, dtype=torch.float64, device=DEV)
    tiles(t_len)
    y = morlet_mix(x, m.plan, m._filters(x.device, torch.float64), a, b)
    (y * gy).sum().backward()
    tiles(0)
    po, ls, w0 = _oracle_inputs(m)
    xo, ao, bo = (t.detach().cpu().requires_grad_() for t in (x, a, b))
    yo = C.mix(xo, po, po.filters(ls.exp(), w0), ao, bo)
    (yo * gy.cpu()).sum().backward()
    close(y, yo, 1e-10, "y")
    for u, v, w in [(x.grad, xo.grad, "dL/dx"), (a.grad, ao.grad, "dL/da"),
                    (b.grad, bo.grad, "dL/db"), (m.log_scales.grad, ls.grad, "dL/dlog_scales"),
                    (m.w0.grad, w0.grad, "dL/dw0")]:
        close(u, v, 1e-10, w)


@pytest.mark.parametrize("per_position", [False, True])
def test_tiled_spectral_softmax_fp64(tiles, per_position):
    torch.manual_seed(6)
    m = F.CWT1D(freqs=np.geomspace(1, 40, 7), fs=200.0, learnable=True,
                learnable_w0=True).to(DEV).double()
    nch, R, N = 3, 6, 1500
    x = torch.randn(R, N, dtype=torch.float64, device=DEV, requires_grad=True)
    shape = (R // nch, 7, N) if per_position else (nch, 7)
    V = torch.randn(shape, dtype=torch.float64, device=DEV, requires_grad=True)
    gy = torch.randn(R, N, dtype=torch.float64, device=DEV)
    tiles(512)
    out = spectral_softmax(x, m.plan, m._filters(x.device, torch.float64), V, nch, 0.8)
    (out * gy).sum().backward()
    tiles(0)
    po, ls, w0 = _oracle_inputs(m)
    xo, Vo = x.detach().cpu().requires_grad_(), V.detach().cpu().requires_grad_()
    oo = C.spectral_softmax(xo, po, po.filters(ls.exp(), w0), Vo, nch, 0.8)
    (oo * gy.cpu()).sum().backward()
    close(out, oo, 1e-10, "out")
    close(x.grad, xo.grad, 1e-10, "dL/dx")
    close(V.grad, Vo.grad, 1e-10, "dL/dV")
    close(m.log_scales.grad, ls.grad, 1e-10, "dL/dlog_scales")
    close(m.w0.grad, w0.grad, 1e-10, "dL/dw0")


def test_long_rows_cwt_64x15000_fwd_bwd():
    """The reference README's CWT shape: 64 rows of 15000 samples, 40 frequencies, learnable,
    forward + backward of sum |W|^2 in fp32, sampled rows against the oracle."""
    torch.manual_seed(7)
    m = F.CWT1D(freqs=np.logspace(-0.3, 2, 40), fs=250.0, norm="l1", learnable=True,
                learnable_w0=True).to(DEV)
    x = torch.randn(64, 15000, device=DEV, requires_grad=True)
    y = m(x)
    torch.view_as_real(y).square().sum().backward()
    rows = [0, 37]
    po, ls, w0 = _oracle_inputs(m)
    xo = x.detach()[rows].double().cpu().requires_grad_()
    yo = C.apply_plan(xo, po, po.filters(ls.exp(), w0))
    yo.abs().square().sum().backward()
    close(y[rows], yo, 1e-4, "W")
    close(x.grad[rows], xo.grad, 1e-4, "dL/dx")
    m.zero_grad()
    torch.view_as_real(m(x.detach()[rows])).square().sum().backward()
    close(m.log_scales.grad, ls.grad, 1e-4, "dL/dlog_scales")
    close(m.w0.grad, w0.grad, 1e-4, "dL/dw0")


def test_long_rows_token_mixer_L16384():
    """MorletTokenMixer at the README's L = 16384 (dim 32, batch 2) in fp32 against the oracle."""
    torch.manual_seed(8)
    mixer = F.MorletTokenMixer(32, freqs=np.logspace(0, 1.8, 16).tolist(), fs=250).to(DEV)
    x = torch.randn(2, 16384, 32, device=DEV, requires_grad=True)
    y = mixer(x)
    y.square().sum().backward()
    cw = mixer.cwt
    po = C.Plan(cw.plan.scales, support_margin=1.25)
    ls = cw.log_scales.detach().double().cpu().requires_grad_()
    P = {k: v.detach().double().cpu().requires_grad_() for k, v in mixer.named_parameters()}
    xo = x.detach()[:1].double().cpu().requires_grad_()
    yo = C.token_mixer(xo, po, po.filters(ls.exp(), cw.w0_value), P["mag_weight"],
                       P["phase_weight"], P["bias"], P["out_proj.weight"], P["out_proj.bias"])
    yo.square().sum().backward()
    close(y[:1], yo, 1e-4, "y")
    close(x.grad[:1], xo.grad, 1e-4, "dL/dx")
    mixer.zero_grad()
    mixer(x.detach()[:1]).square().sum().backward()
    close(cw.log_scales.grad, ls.grad, 1e-4, "dL/dlog_scales")
    close(mixer.mag_weight.grad, P["mag_weight"].grad, 1e-4, "dL/dmag_weight")
