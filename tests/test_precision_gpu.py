"""The reference's precision switches (``fdwt.config.allow_tf32`` / ``allow_bf16``,
``fdwt/config.py:17-18``) and its reduced-precision tolerance tests
(``tests/test_dwt.py:75-85``, ``tests/test_cwt.py:103-113``).

In the reference the switches let its Triton dots take TF32 or bf16 operands
(``kernels/conv.py:332-338``).  These kernels compute every filter-bank contraction with fp32
FMAs (fp64 for fp64 rows), so the switches grant a precision they never need: with either
switch on, every transform and layer output must be bit-identical to the switch-off result
(gradients too, up to the run-to-run rounding of atomic sums), and so within the reference's
tolerances for those modes (TF32 / bf16 dots: 1e-2 and 6e-2 relative) and its fp32 bar (1e-5).
"""

import numpy as np
import pytest
import torch

import pytorch_morlet_fdwt_b200 as F
from pytorch_morlet_fdwt_b200 import config

pytestmark = pytest.mark.gpu
DEV = "cuda"
FREQS = np.geomspace(0.5, 100, 24)
FLAGS = [("allow_tf32", True), ("allow_bf16", True)]


@pytest.fixture
def flag():
    saved = (config.allow_tf32, config.allow_bf16)

    def set_flag(name, value):
        config.allow_tf32, config.allow_bf16 = saved
        if name is not None:
            setattr(config, name, value)

    yield set_flag
    config.allow_tf32, config.allow_bf16 = saved


def rel(a, b):
    a, b = a.detach(), b.detach()
    if a.is_complex():
        a, b = torch.view_as_real(a), torch.view_as_real(b)
    return float((a.double() - b.double()).abs().max() / b.double().abs().max())


@pytest.mark.parametrize("name,value", FLAGS)
def test_dwt_under_precision_switches(flag, name, value):
    torch.manual_seed(0)
    x = torch.randn(4, 1000, device=DEV)
    ref = F.wavedec(x.double(), "db4", level=4)
    flag(None, None)
    base = {dt: F.wavedec(x.to(dt), "db4", level=4)
            for dt in (torch.float32, torch.float16, torch.bfloat16)}
    flag(name, value)
    for dt, tol in ((torch.float32, 1e-5), (torch.float16, 1e-2), (torch.bfloat16, 6e-2)):
        out = F.wavedec(x.to(dt), "db4", level=4)
        for o, b, r in zip(out, base[dt], ref):
            assert o.dtype == dt
            assert torch.equal(o, b)
            assert rel(o, r) <= tol
        y = F.waverec(out, "db4")
        assert y.dtype == dt


@pytest.mark.parametrize("name,value", FLAGS)
def test_cwt_under_precision_switches(flag, name, value):
    torch.manual_seed(0)
    x = torch.randn(8, 2500, device=DEV)
    ref = F.cwt(x.double(), freqs=FREQS, fs=250, method="fast")
    flag(None, None)
    base32 = F.cwt(x, freqs=FREQS, fs=250, method="fast")
    base16 = F.cwt(x.half(), freqs=FREQS, fs=250, method="fast")
    flag(name, value)
    out = F.cwt(x, freqs=FREQS, fs=250, method="fast")
    out16 = F.cwt(x.half(), freqs=FREQS, fs=250, method="fast")
    assert out.dtype == torch.complex64 and out16.dtype == torch.complex64
    assert torch.equal(out, base32) and torch.equal(out16, base16)
    assert rel(out, ref) < 1e-5
    assert rel(out16, ref) < 1e-2


def _layer_step(m, x):
    m.zero_grad()
    x = x.detach().clone().requires_grad_()
    y = m(x)
    (y * torch.linspace(-1, 1, y.numel(), device=DEV).view_as(y)).sum().backward()
    return [y.detach(), x.grad] + [p.grad.clone() for p in m.parameters() if p.grad is not None]


@pytest.mark.parametrize("name,value", FLAGS)
def test_layers_under_precision_switches(flag, name, value):
    torch.manual_seed(1)
    layers = [
        (F.MorletTokenMixer(32, freqs=np.logspace(0, 1.8, 16).tolist(), fs=250).to(DEV),
         torch.randn(2, 600, 32, device=DEV)),
        (F.MorletAttention(3, 50).to(DEV), torch.randn(2, 2, 3, 4, 50, device=DEV)),
        (F.MorletChannelMixAttention(3, 50).to(DEV), torch.randn(2, 2, 3, 4, 50, device=DEV)),
    ]
    for m, x in layers:
        flag(None, None)
        base = _layer_step(m, x)
        flag(name, value)
        got = _layer_step(m, x)
        assert len(got) == len(base)
        assert torch.equal(got[0], base[0])
        # the channel mix's per-position dL/dU sums the C rows of a group with atomic adds, so
        # its gradients can differ from run to run in the last bits
        for g, b in zip(got[1:], base[1:]):
            assert rel(g, b) <= 1e-6
