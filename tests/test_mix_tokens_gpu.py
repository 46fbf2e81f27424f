"""The mix on MorletTokenMixer's token layout (fdwt_mix_tokens_forward / _backward): the kernels
read x (B, L, D) and write y + bias (B, L, D) themselves, and the backward takes dL/dy and
returns dL/dx in that layout, where the reference transposes around ``morlet_mix`` and adds the
bias in separate kernels (``fdwt/layers.py:49-55``).

* Against the row-layout path (``morlet_mix`` on ``x.transpose(1, 2)``, the reference's own
  glue): y and every gradient are bit-identical (the kernels do the same arithmetic per row),
  except dL/dbias, a sum in another order (1e-12 in fp64).
* On whole rows and on time tiles (forced, and rows longer than one CTA's shared memory).
* gradcheck / gradgradcheck of the token-layout Function in fp64, bias included.
"""

import numpy as np
import pytest
import torch
from torch.autograd import gradcheck, gradgradcheck

import pytorch_morlet_fdwt_b200 as F
from pytorch_morlet_fdwt_b200 import _lib
from pytorch_morlet_fdwt_b200.cwt import morlet_mix, morlet_mix_tokens

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture
def tiles():
    yield _lib.set_cwt_tile_test
    _lib.set_cwt_tile_test(0)


def _run(fn, x, H, a, b, bias, gy):
    x = x.detach().clone().requires_grad_()
    H = H.detach().clone().requires_grad_()
    a = a.detach().clone().requires_grad_()
    b = b.detach().clone().requires_grad_()
    bias = bias.detach().clone().requires_grad_()
    y = fn(x, H, a, b, bias)
    (y * gy).sum().backward()
    return y.detach(), x.grad, H.grad, a.grad, b.grad, bias.grad


CASES = [
    # (B, L, D, freqs, dtype, forced tile)
    (2, 600, 24, np.logspace(0, 1.8, 16), torch.float32, 0),
    (3, 257, 5, np.logspace(0.3, 2.0, 9), torch.float64, 0),
    (2, 1500, 8, np.logspace(0, 1.8, 16), torch.float32, 320),
    (1, 16384, 3, np.logspace(0, 1.8, 16), torch.float32, 0),
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_tokens_match_row_layout(tiles, case):
    B, L, D, freqs, dt, tile = CASES[case]
    torch.manual_seed(case)
    m = F.CWT1D(freqs=freqs, fs=250.0, learnable=True).to(DEV)
    H = m._filters(DEV, dt).detach()
    x = torch.randn(B, L, D, device=DEV, dtype=dt)
    a = torch.randn(D, len(freqs), device=DEV, dtype=dt)
    b = torch.randn(D, len(freqs), device=DEV, dtype=dt)
    bias = torch.randn(D, device=DEV, dtype=dt)
    gy = torch.randn(B, L, D, device=DEV, dtype=dt)
    tiles(tile)
    tok = _run(lambda x, H, a, b, c: morlet_mix_tokens(x, m.plan, H, a, b, c), x, H, a, b, bias, gy)
    row = _run(lambda x, H, a, b, c: morlet_mix(x.transpose(1, 2), m.plan, H, a, b)
               .transpose(1, 2) + c, x, H, a, b, bias, gy)
    for name, u, v in zip(("y", "dx", "dH", "da", "db"), tok[:5], row[:5]):
        assert torch.equal(u, v), name
    err = float((tok[5] - row[5]).abs().max() / row[5].abs().max())
    assert err <= (1e-12 if dt == torch.float64 else 1e-6), err


def test_tokens_without_bias_and_noncontiguous_input():
    torch.manual_seed(7)
    m = F.CWT1D(freqs=np.logspace(0, 1.8, 16), fs=250.0).to(DEV)
    H = m._filters(DEV, torch.float32)
    xt = torch.randn(2, 12, 700, device=DEV)  # (B, D, L): the tokens are its transpose
    a = torch.randn(12, 16, device=DEV)
    b = torch.randn(12, 16, device=DEV)
    y = morlet_mix_tokens(xt.transpose(1, 2), m.plan, H, a, b)
    ref = morlet_mix(xt, m.plan, H, a, b).transpose(1, 2)
    assert torch.equal(y, ref)


def test_token_mixer_layer_matches_row_glue():
    """MorletTokenMixer (token kernels) against the reference's glue on the row kernels."""
    torch.manual_seed(0)
    m = F.MorletTokenMixer(32, freqs=np.logspace(0, 1.8, 16).tolist(), fs=250).to(DEV)
    with torch.no_grad():
        m.bias.normal_()
    x = torch.randn(3, 900, 32, device=DEV, requires_grad=True)
    y = m(x)
    y.square().sum().backward()
    got = [y.detach(), x.grad.clone()] + [p.grad.clone() for p in m.parameters()]
    m.zero_grad()
    x.grad = None
    H = m.cwt._filters(DEV, torch.float32)
    y2 = morlet_mix(x.transpose(1, 2), m.cwt.plan, H, m.mag_weight, m.phase_weight)
    y2 = m.out_proj(y2.transpose(1, 2) + m.bias)
    y2.square().sum().backward()
    ref = [y2.detach(), x.grad.clone()] + [p.grad.clone() for p in m.parameters()]
    names = ["y", "dx"] + [n for n, _ in m.named_parameters()]
    for name, u, v in zip(names, got, ref):
        tol = 1e-6 if name == "bias" else 0.0
        err = float((u - v).abs().max() / v.abs().max().clamp_min(1e-30))
        assert err <= tol, (name, err)


def test_gradcheck_tokens_fp64():
    torch.manual_seed(2)
    m = F.CWT1D(scales=[1.5, 4.0, 11.0], learnable=True, learnable_w0=True).to(DEV).double()
    x = torch.randn(2, 40, 3, dtype=torch.float64, device=DEV, requires_grad=True)
    a = torch.randn(3, 3, dtype=torch.float64, device=DEV, requires_grad=True)
    b = torch.randn(3, 3, dtype=torch.float64, device=DEV, requires_grad=True)
    c = torch.randn(3, dtype=torch.float64, device=DEV, requires_grad=True)
    ls = m.log_scales.detach().clone().requires_grad_()

    def f(x, a, b, c, ls):
        return morlet_mix_tokens(x, m.plan, m.plan.filters(ls.exp(), 6.0, torch.float64), a, b, c)

    assert gradcheck(f, (x, a, b, c, ls))
    assert gradgradcheck(f, (x, a, b, c, ls))
