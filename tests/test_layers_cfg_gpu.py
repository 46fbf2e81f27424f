"""The fused layers and the learnable CWT at the baseline configs' own shapes, in fp32 on the
GPU (sm_100a kernels through the C ABI), against the fp64 CPU oracle.

* ``MorletTokenMixer(256, freqs=logspace(0, 1.8, 16), fs=250)`` on x (8, 4096, 256);
* ``MorletAttention`` and ``MorletChannelMixAttention`` with 19 channels, hidden 200,
  on x (64, 4, 19, 30, 200);
* configs[2] with learnable scales and w0: the filter gradient of all 2048 rows.

Each layer is built right after ``torch.manual_seed(0)``, as the reference's benchmarks build
theirs (parameters draw from that generator), and runs forward plus the backward of
``y.square().sum()`` on the full batch.  The loss is a sum over batch entries, so the output and
dL/dx of any batch entry depend on that entry alone: sampled entries are compared with the
oracle run on just those entries.  Parameter gradients are sums over the batch: they are
compared on a GPU run over the same sampled entries.

Tolerance: 1e-4 x max|ref| (the bound stated for CWT, mixer outputs and gradients in fp32).
"""

import numpy as np
import pytest
import torch

import pytorch_morlet_fdwt_b200 as F
from oracle import cwt_oracle as C

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-4


def close(a, b, tol=TOL, what=""):
    a = a.detach().cpu().double()
    b = b.detach().cpu().double()
    assert a.shape == b.shape, (what, a.shape, b.shape)
    scale = float(b.abs().max())
    err = float((a - b).abs().max())
    assert err <= tol * max(scale, 1e-300), f"{what}: max err {err:.3e} > {tol:.1e} x {scale:.3e}"


def _oracle_filters(cwt_mod):
    """fp64 oracle plan and differentiable filter inputs matching a CWT1D module."""
    po = C.Plan(cwt_mod.plan.scales, w0=cwt_mod.plan.w0, truncate=cwt_mod.plan.truncate,
                norm=cwt_mod.plan.norm, complex=cwt_mod.plan.complex,
                support_margin=1.25 if cwt_mod._learn else 1.0)
    ls = cwt_mod.log_scales.detach().double().cpu().requires_grad_(cwt_mod._learn)
    if isinstance(cwt_mod.w0, torch.Tensor):
        w0 = cwt_mod.w0.detach().double().cpu().requires_grad_()
    else:
        w0 = cwt_mod.w0
    return po, ls, w0


def _cpu_params(mod):
    return {k: v.detach().double().cpu().requires_grad_() for k, v in mod.named_parameters()
            if v.requires_grad}


def test_cfg4_token_mixer_fp32_vs_oracle():
    torch.manual_seed(0)
    m = F.MorletTokenMixer(256, freqs=np.logspace(0, 1.8, 16).tolist(), fs=250).to(DEV)
    x = torch.randn(8, 4096, 256, device=DEV, requires_grad=True)
    y = m(x)
    y.square().sum().backward()
    assert torch.isfinite(x.grad).all()
    pick = [0, 5]
    po, ls, w0 = _oracle_filters(m.cwt)
    P = _cpu_params(m)
    xs = x.detach()[pick].double().cpu().requires_grad_()
    yo = C.token_mixer(xs, po, po.filters(ls.exp(), w0), P["mag_weight"], P["phase_weight"],
                       P["bias"], P["out_proj.weight"], P["out_proj.bias"])
    yo.square().sum().backward()
    close(y[pick], yo, what="y")
    close(x.grad[pick], xs.grad, what="dL/dx")
    # parameter gradients of the same two entries, from the GPU
    m.zero_grad()
    m(x.detach()[pick]).square().sum().backward()
    close(m.cwt.log_scales.grad, ls.grad, what="log_scales")
    for name in ("mag_weight", "phase_weight", "bias", "out_proj.weight", "out_proj.bias"):
        close(dict(m.named_parameters())[name].grad, P[name].grad, what=name)


@pytest.mark.parametrize("channel_mix", [False, True])
def test_cfg5_attention_fp32_vs_oracle(channel_mix):
    cls = F.MorletChannelMixAttention if channel_mix else F.MorletAttention
    torch.manual_seed(0)
    m = cls(num_channels=19, hidden_dim=200).to(DEV)
    x = torch.randn(64, 4, 19, 30, 200, device=DEV, requires_grad=True)
    y = m(x)
    y.square().sum().backward()
    assert torch.isfinite(x.grad).all()
    pick = [0, 41]
    po, ls, w0 = _oracle_filters(m.cwt)
    P = _cpu_params(m)
    xs = x.detach()[pick].double().cpu().requires_grad_()
    H = po.filters(ls.exp(), w0)
    if channel_mix:
        yo = C.channel_mix_attention(xs, po, H, P["freq_to_channel"], m.temperature)
    else:
        yo = C.attention(xs, po, H, P["freq_weight"], m.temperature)
    yo.square().sum().backward()
    close(y[pick], yo, what="y")
    close(x.grad[pick], xs.grad, what="dL/dx")
    m.zero_grad()
    m(x.detach()[pick]).square().sum().backward()
    close(m.cwt.log_scales.grad, ls.grad, what="log_scales")
    close(m.cwt.w0.grad, w0.grad, what="w0")
    name = "freq_to_channel" if channel_mix else "freq_weight"
    close(dict(m.named_parameters())[name].grad, P[name].grad, what=name)


def test_cfg3_learnable_filter_gradient_all_rows():
    """dL/dlog_scales and dL/dw0 of all 2048 rows of configs[2] (learnable): the full-batch GPU
    gradient equals the sum of the GPU gradients of four 512-row subsets, and two of those
    subsets are compared with the fp64 oracle on a 16-row sample each (the gradient is a sum
    over rows: each subset's is the sum of its rows')."""
    torch.manual_seed(3)
    m = F.CWT1D(freqs=np.logspace(-0.3, 2, 40), fs=250.0, norm="l1", learnable=True,
                learnable_w0=True).to(DEV)
    x = torch.randn(2048, 2500, device=DEV)

    def grads(rows):
        m.zero_grad()
        torch.view_as_real(m(rows)).square().sum().backward()
        return m.log_scales.grad.double().clone(), m.w0.grad.double().clone()

    full_ls, full_w0 = grads(x)
    parts = [grads(x[i:i + 512]) for i in range(0, 2048, 512)]
    # the same sums in another fp32 order: 1e-4, the fp32 gradient bound
    close(full_ls, sum(p[0] for p in parts), what="all rows vs subsets (log_scales)")
    close(full_w0, sum(p[1] for p in parts), what="all rows vs subsets (w0)")
    po, _, _ = _oracle_filters(m)
    for start in (0, 1536):
        rows = x[start:start + 16]
        g_ls, g_w0 = grads(rows)
        ls = m.log_scales.detach().double().cpu().requires_grad_()
        w0 = m.w0.detach().double().cpu().requires_grad_()
        W = C.apply_plan(rows.double().cpu(), po, po.filters(ls.exp(), w0))
        W.abs().square().sum().backward()
        close(g_ls, ls.grad, what=f"log_scales rows {start}+16")
        close(g_w0, w0.grad, what=f"w0 rows {start}+16")
