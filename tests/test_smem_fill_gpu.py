"""No output may depend on uninitialised shared memory.

Shared memory is not cleared between kernels, so a cell that a kernel reads without having
written it holds whatever an earlier kernel left there -- finite values most of the time, which
hides the read when it only feeds a zero tap (0 * x = 0), but 0 * inf and 0 * nan are nan.  With
the library's test hook fdwt_set_shared_memory_fill on, every kernel of the library is preceded
by one that sets all shared memory to a NaN (or -inf) bit pattern; the transforms, their
backward passes and the fused CWT epilogues must then still match the CPU oracle (DWT) or the
same calls without the fill (CWT, mix, spectral softmax), at the same tolerances as the parity
tests.  The DWT cases cover the tile synthesis unsplit over 4, 6 and 8 levels with several tiles
per row (the periodization cases of 6 and 8 levels read, before every margin cell of the
approximation segments was zeroed, cells through zero taps that no level had written), split
into coarse and fine launches, and with every level whole in one tile; the cluster analysis in
one and several segments; every boundary mode.
"""

import numpy as np
import pytest
import torch

import pytorch_morlet_fdwt_b200 as F
from pytorch_morlet_fdwt_b200 import _lib
from pytorch_morlet_fdwt_b200.cwt import morlet_mix, spectral_softmax
from oracle import dwt_oracle as D

pytestmark = pytest.mark.gpu
DEV = "cuda"
FILLS = {"nan": 0xFFFFFFFF, "neg_inf_f32": 0xFF800000}  # 0xFFFFFFFF is a NaN in fp32 and fp64


@pytest.fixture
def fill():
    yield lambda word: _lib.set_shared_memory_fill(True, word)
    torch.cuda.synchronize()
    _lib.set_shared_memory_fill(False)


def close(a, b, tol):
    a = a.detach().double().cpu().numpy() if torch.is_tensor(a) else np.asarray(a)
    b = b.detach().double().cpu().numpy() if torch.is_tensor(b) else np.asarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    assert np.isfinite(a).all(), "non-finite output"
    scale = max(1e-300, float(np.abs(b).max()) if b.size else 1.0)
    err = float(np.abs(a - b).max()) if b.size else 0.0
    assert err <= tol * scale, f"max err {err:.3e} > {tol:.1e} x {scale:.3e}"


# (dtype, rows, n, wavelet, mode, level, tolerance)
DWT_CASES = [
    (torch.float32, 4, 65536, "db8", "periodization", 4, 1e-5),
    (torch.float32, 4, 65536, "db8", "symmetric", 8, 1e-5),
    (torch.float32, 4, 65536, "db4", "zero", 5, 1e-5),
    (torch.float64, 2, 32768, "db4", "reflect", 6, 1e-12),
    (torch.float64, 2, 20000, "db20", "periodic", 4, 1e-12),
    (torch.bfloat16, 4, 65536, "db8", "symmetric", 8, 6e-2),
    (torch.bfloat16, 4, 65536, "db8", "periodization", 8, 6e-2),
    (torch.float32, 16, 8000, "db8", "periodization", 6, 1e-5),
    (torch.float64, 16, 4000, "db4", "periodization", 6, 1e-12),
    (torch.float32, 64, 2500, "db4", "symmetric", 5, 1e-5),
    (torch.float32, 8, 9000, "haar", "periodization", 6, 1e-5),
]


@pytest.mark.parametrize("word", list(FILLS.values()), ids=list(FILLS))
@pytest.mark.parametrize("case", DWT_CASES,
                         ids=[f"{str(c[0])[6:]}-{c[1]}x{c[2]}-{c[3]}-{c[4]}-L{c[5]}"
                              for c in DWT_CASES])
def test_dwt_ignores_uninitialised_shared_memory(case, word, fill):
    dtype, rows, n, wname, mode, level, tol = case
    torch.manual_seed(3)
    bank = F.get_filter_bank(wname)
    tb = (bank.dec_lo, bank.dec_hi, bank.rec_lo, bank.rec_hi)
    x = torch.randn(rows, n, device=DEV).to(dtype)
    ref = D.wavedec(x.double().cpu().numpy(), tb, mode, level)
    yref = D.waverec(ref, tb, mode)
    gx_ref = D.wavedec_vjp(n, [2 * r for r in ref], tb, mode)
    gy = torch.randn(yref.shape, device=DEV).to(dtype)
    gc_ref = D.waverec_vjp(ref, gy.double().cpu().numpy(), tb, mode)

    fill(word)
    xg = x.clone().requires_grad_()
    coeffs = F.wavedec(xg, bank, mode, level)
    sum((c.double() ** 2).sum() for c in coeffs).backward()
    cg = [c.detach().clone().requires_grad_() for c in coeffs]
    y = F.waverec(cg, bank, mode)
    (y.double() * gy.double()).sum().backward()
    torch.cuda.synchronize()

    for c, r in zip(coeffs, ref):
        close(c, r, tol)
    close(xg.grad, gx_ref, tol)
    close(y, yref, tol)
    for c, r in zip(cg, gc_ref):
        close(c.grad, r, tol)


def _cwt_family(dtype, x, a, b, V, gm, gs):
    """CWT forward + backward (x, scales, w0), the fused mix and the spectral softmax with
    their backward passes; returns every output and gradient."""
    torch.manual_seed(7)
    m = F.CWT1D(freqs=np.geomspace(0.5, 100, 40), fs=250.0, norm="l1", learnable=True,
                learnable_w0=True).to(DEV).to(dtype)
    outs = []
    xx = x.clone().requires_grad_()
    W = m(xx)
    W.abs().square().sum().backward()
    outs += [W, xx.grad, m.log_scales.grad, m.w0.grad]
    m.zero_grad()
    H = m.plan.filters(m.log_scales.exp(), m.w0, dtype)
    xm = x.view(2, 3, -1).clone().requires_grad_()
    aa, bb = a.clone().requires_grad_(), b.clone().requires_grad_()
    y = morlet_mix(xm, m.plan, H, aa, bb)
    (y * gm).sum().backward()
    outs += [y, xm.grad, aa.grad, bb.grad, m.log_scales.grad, m.w0.grad]
    m.zero_grad()
    H = m.plan.filters(m.log_scales.exp(), m.w0, dtype)
    xs = x.clone().requires_grad_()
    VV = V.clone().requires_grad_()
    o = spectral_softmax(xs, m.plan, H, VV, 3, 0.7)
    (o * gs).sum().backward()
    outs += [o, xs.grad, VV.grad, m.log_scales.grad, m.w0.grad]
    return [t.detach() for t in outs]


@pytest.mark.parametrize("word", list(FILLS.values()), ids=list(FILLS))
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.float64, 1e-12)])
def test_cwt_mix_softmax_ignore_uninitialised_shared_memory(dtype, tol, word, fill):
    torch.manual_seed(5)
    x = torch.randn(6, 2500, device=DEV, dtype=dtype)
    a = torch.randn(3, 40, device=DEV, dtype=dtype)
    b = torch.randn(3, 40, device=DEV, dtype=dtype)
    V = torch.randn(3, 40, device=DEV, dtype=dtype)
    gm = torch.randn(2, 3, 2500, device=DEV, dtype=dtype)
    gs = torch.randn(6, 2500, device=DEV, dtype=dtype)
    base = _cwt_family(dtype, x, a, b, V, gm, gs)
    fill(word)
    got = _cwt_family(dtype, x, a, b, V, gm, gs)
    torch.cuda.synchronize()
    for g, r in zip(got, base):
        if g.is_complex():
            g, r = torch.view_as_real(g), torch.view_as_real(r)
        close(g, r, tol)
