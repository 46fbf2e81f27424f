"""WaveletTokenMixer and MorletChannelMixAttention.attention_map on the GPU against the CPU
oracle (fp64).

* ``WaveletTokenMixer`` (``fdwt/layers.py:75-109``): multilevel DWT of the token axis through
  the sm_100a kernels, a per-band Linear over the channels, inverse DWT; compared with the
  oracle's sparse-operator DWT (``oracle/dwt_oracle.py``) and the same Linear layers in numpy,
  output and dL/dx.
* ``attention_map`` (``fdwt/layers.py:252-255``): the explicit (B, H, N, C, C) map from the
  softmax over frequencies of |W| and the frequency-to-channel matrix.

Tolerance 1e-10 x max|ref| (fp64).
"""

import numpy as np
import pytest
import torch

import pytorch_morlet_fdwt_b200 as F
from oracle import cwt_oracle as C
from oracle import dwt_oracle as D

pytestmark = pytest.mark.gpu
DEV = "cuda"


def close(a, b, tol=1e-10, what=""):
    a = a.detach().cpu().double().numpy() if torch.is_tensor(a) else np.asarray(a)
    b = b.detach().cpu().double().numpy() if torch.is_tensor(b) else np.asarray(b)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    scale = float(np.abs(b).max())
    err = float(np.abs(a - b).max())
    assert err <= tol * max(scale, 1e-300), f"{what}: max err {err:.3e} > {tol:.1e} x {scale:.3e}"


@pytest.mark.parametrize("mode,level,hidden", [("periodization", 3, 0), ("symmetric", 2, 0),
                                               ("periodization", 2, 12)])
def test_wavelet_token_mixer_vs_oracle(mode, level, hidden):
    torch.manual_seed(0)
    B, L, Dm = 2, 96, 8
    m = F.WaveletTokenMixer(Dm, "db4", mode, level, hidden).double()
    x = torch.randn(B, L, Dm, dtype=torch.float64)
    xg = x.to(DEV).requires_grad_()
    mg = m.to(DEV)
    y = mg(xg)
    gy = torch.randn_like(y)
    (y * gy).sum().backward()

    bank = F.get_filter_bank("db4")
    tb = (bank.dec_lo, bank.dec_hi, bank.rec_lo, bank.rec_hi)
    rows = x.transpose(1, 2).reshape(B * Dm, L).numpy()
    coeffs = D.wavedec(rows, tb, mode, level)
    cpu_bands = [band.cpu() for band in m.bands]

    def apply_band(band, c):  # c (B*D, n) -> (B*D, n), Linear over the channel axis
        t = torch.from_numpy(c).view(B, Dm, -1).transpose(1, 2).requires_grad_()
        out = band(t).transpose(1, 2).reshape(B * Dm, -1)
        return t, out

    ins, outs = [], []
    for band, c in zip(cpu_bands, coeffs):
        t, o = apply_band(band, c)
        ins.append(t)
        outs.append(o)
    yr = D.waverec([o.detach().numpy() for o in outs], tb, mode)[:, :L]
    yo = torch.from_numpy(yr).view(B, Dm, L).transpose(1, 2)
    close(y, yo, what="y")
    # dL/dx: waverec's vjp, the bands' backward, wavedec's vjp
    gyr = gy.cpu().transpose(1, 2).reshape(B * Dm, L).numpy()
    full = np.zeros((B * Dm, D.waverec([o.detach().numpy() for o in outs], tb, mode).shape[1]))
    full[:, :L] = gyr
    gouts = D.waverec_vjp([o.detach().numpy() for o in outs], full, tb, mode)
    gcoef = []
    for t, o, g in zip(ins, outs, gouts):
        (gt,) = torch.autograd.grad(o, t, torch.from_numpy(np.ascontiguousarray(g)))
        gcoef.append(gt.transpose(1, 2).reshape(B * Dm, -1).numpy())
    gx = D.wavedec_vjp(L, gcoef, tb, mode).reshape(B, Dm, L).transpose(0, 2, 1)
    close(xg.grad, gx, what="dL/dx")


def test_attention_map_vs_oracle():
    torch.manual_seed(1)
    m = F.MorletChannelMixAttention(num_channels=3, hidden_dim=40, temperature=0.7).double()
    x = torch.randn(1, 2, 3, 4, 40, dtype=torch.float64)
    amap = m.to(DEV).attention_map(x.to(DEV))
    po = C.Plan(m.cwt.plan.scales, support_margin=1.25)
    H = po.filters(m.cwt.log_scales.detach().cpu().double().exp(),
                   m.cwt.w0.detach().cpu().double())
    w = C.apply_plan(x.reshape(1, 2, 3, 160), po, H)            # (B, H, C, f, N)
    p = torch.softmax(w.abs() / 0.7, dim=-2)
    ref = torch.einsum("bhcfn,fk->bhnck", p, m.freq_to_channel.detach().cpu().double())
    close(amap, ref, what="attention_map")
