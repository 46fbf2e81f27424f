"""Generate the golden fixtures from the reference's own CPU path.

Run in the build container, where the reference source tree is mounted:

    python tests/golden/make_golden.py --reference-src <path to pytorch_morlet_fdwt>/src

It imports the reference package (``fdwt``), feeds it seeded fp64 CPU tensors (which selects
its pure-PyTorch CPU path: ``fdwt/dwt.py:23-24``, ``fdwt/cwt.py:386, 539, 605``) and stores
inputs, outputs and autograd gradients in ``tests/golden/*.npz``.  PyWavelets is absent here,
so every DWT case passes an explicit filter bank (Daubechies banks from
``pytorch_morlet_fdwt_b200.wavelets.daubechies_scaling_filter`` plus a random custom bank);
the banks are stored with the fixtures.  The fixtures are what pins the CPU oracle in
``oracle/``; the GPU tests then compare the CUDA kernels against that oracle and these files.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from pytorch_morlet_fdwt_b200.wavelets import daubechies_scaling_filter  # noqa: E402

MODES = ["zero", "periodic", "symmetric", "reflect", "periodization"]


def orthogonal_bank(order):
    h = daubechies_scaling_filter(order)
    L = len(h)
    rec_lo = list(h)
    rec_hi = [(-1) ** k * h[L - 1 - k] for k in range(L)]
    return (rec_lo[::-1], rec_hi[::-1], rec_lo, rec_hi)


def banks():
    g = np.random.default_rng(7)
    custom = tuple(list(g.standard_normal(5)) for _ in range(4))  # odd length: padded to 6
    return {"haar": orthogonal_bank(1), "db2": orthogonal_bank(2), "db4": orthogonal_bank(4),
            "db8": orthogonal_bank(8), "rand5": custom}


def np64(t):
    return t.detach().cpu().numpy().astype(np.float64)


def dwt_single(fdwt, out):
    B = banks()
    torch.manual_seed(0)
    for bname in ["haar", "db2", "db4", "rand5"]:
        bank = B[bname]
        for mode in MODES:
            for n in [1, 2, 3, 7, 16, 33, 100]:
                x = torch.randn(2, n, dtype=torch.float64)
                key = f"{bname}|{mode}|{n}"
                a, d = fdwt.dwt(x, bank, mode)
                out[key + "|x"], out[key + "|a"], out[key + "|d"] = np64(x), np64(a), np64(d)
                try:
                    y = fdwt.idwt(a, d, bank, mode)
                    out[key + "|y"] = np64(y)
                except ValueError:
                    pass
                # gradients of a fixed quadratic loss through dwt and idwt
                xg = x.clone().requires_grad_()
                a2, d2 = fdwt.dwt(xg, bank, mode)
                (a2.square().sum() + 3.0 * d2.square().sum()).backward()
                out[key + "|gx"] = np64(xg.grad)
                if key + "|y" in out:
                    ag, dg = a.clone().requires_grad_(), d.clone().requires_grad_()
                    fdwt.idwt(ag, dg, bank, mode).square().sum().backward()
                    out[key + "|ga"], out[key + "|gd"] = np64(ag.grad), np64(dg.grad)
    for bname, bank in B.items():
        for i, f in enumerate(bank):
            out[f"bank|{bname}|{i}"] = np.asarray(f, dtype=np.float64)


def dwt_multi(fdwt, out):
    B = banks()
    torch.manual_seed(1)
    cases = [(b, m, n, 1) for b in ["db4", "db8"] for m in MODES for n in [64, 517]]
    cases += [("db4", "symmetric", 2500, 3), ("db8", "periodization", 4096, 1),
              ("db4", "reflect", 1, 1), ("db2", "periodization", 7, 2)]
    for bname, mode, n, rows in cases:
        bank = B[bname]
        x = torch.randn(rows, n, dtype=torch.float64)
        key = f"{bname}|{mode}|{n}"
        lvl = 5 if n == 2500 else (3 if n <= 7 else None)
        xg = x.clone().requires_grad_()
        coeffs = fdwt.wavedec(xg, bank, mode, lvl)
        sum((c.square() * (1.0 + i)).sum() for i, c in enumerate(coeffs)).backward()
        out[key + "|x"] = np64(x)
        out[key + "|level"] = np.array(len(coeffs) - 1)
        out[key + "|gx"] = np64(xg.grad)
        cs = [c.detach().clone().requires_grad_() for c in coeffs]
        for i, c in enumerate(cs):
            out[key + f"|c{i}"] = np64(c)
        y = fdwt.waverec(cs, bank, mode)
        y.square().sum().backward()
        out[key + "|y"] = np64(y)
        for i, c in enumerate(cs):
            out[key + f"|gc{i}"] = np64(c.grad)


def plan_record(fdwt, out, key, scales, **kw):
    p = fdwt.MorletPlan(scales, **kw)
    out[key + "|scales"] = np.asarray(scales, dtype=np.float64)
    out[key + "|margins"] = np.asarray(p.margins, dtype=np.int64)
    out[key + "|meta"] = np.array([p.n_octaves, p.center, p.c_lp], dtype=np.int64)
    out[key + "|lowpass"] = p.lowpass.numpy()
    for k, st in enumerate(p.stages):
        out[key + f"|stage{k}"] = np.array([st.octave, st.dil, st.half] + st.scale_idx + st.support,
                                           dtype=np.int64)
    s = torch.tensor(p.scales, dtype=torch.float64)
    out[key + "|filters"] = p.filters(s, p.w0, torch.float64).numpy()


def cwt_cases(fdwt, out):
    fs = 250.0
    f = fdwt.freqs_to_scales
    plan_record(fdwt, out, "plan|cfg3", f(np.logspace(-0.3, 2, 40), fs).tolist(), norm="l1")
    plan_record(fdwt, out, "plan|cfg3l", f(np.logspace(-0.3, 2, 40), fs).tolist(), norm="l1",
                support_margin=1.25)
    plan_record(fdwt, out, "plan|cfg4", f(np.logspace(0, 1.8, 16), fs).tolist(), support_margin=1.25)
    plan_record(fdwt, out, "plan|cfg5", f(np.logspace(0, np.log10(40.0), 16), 200.0).tolist(),
                support_margin=1.25)
    plan_record(fdwt, out, "plan|t5", f(np.geomspace(0.5, 100, 24), fs).tolist(), truncate=5.0)
    plan_record(fdwt, out, "plan|w0", [1.2, 3.0, 7.0, 40.0, 90.0], w0=2.0, norm="l1")
    plan_record(fdwt, out, "plan|direct", f(np.geomspace(1, 60, 8), fs).tolist(), method="direct")

    torch.manual_seed(2)
    freqs = np.geomspace(1, 60, 8)
    x = torch.randn(2, 500, dtype=torch.float64)
    out["cwt|x"] = np64(x)
    for method, norm, cplx, trunc in [("fast", "l1", True, 4.0), ("fast", "l2", False, 4.0),
                                      ("direct", "l2", True, 4.0), ("fast", "l2", True, 5.0)]:
        y = fdwt.cwt(x, freqs=freqs, fs=fs, method=method, norm=norm, complex=cplx, truncate=trunc)
        y = torch.view_as_real(y) if cplx else y
        out[f"cwt|{method}|{norm}|{int(cplx)}|{trunc:g}"] = np64(y)

    torch.manual_seed(3)
    xl = torch.randn(2, 400, dtype=torch.float64)
    for cplx in (True, False):
        m = fdwt.CWT1D(freqs=freqs[:6], fs=fs, learnable=True, learnable_w0=True, complex=cplx).double()
        xx = xl.clone().requires_grad_()
        y = m(xx)
        (y.abs().square().sum() if cplx else (y.square() * y.new_tensor(1.5)).sum()).backward()
        key = f"cwtlearn|{int(cplx)}"
        out[key + "|x"] = np64(xl)
        out[key + "|gx"] = np64(xx.grad)
        out[key + "|gls"] = np64(m.log_scales.grad)
        out[key + "|gw0"] = np64(m.w0.grad)


def layer_cases(fdwt, out):
    torch.manual_seed(4)
    mixer = fdwt.MorletTokenMixer(8, freqs=np.geomspace(1, 40, 6).tolist(), fs=250).double()
    x = torch.randn(2, 300, 8, dtype=torch.float64)
    xx = x.clone().requires_grad_()
    y = mixer(xx)
    y.square().sum().backward()
    k = "mixer"
    out[k + "|x"], out[k + "|y"], out[k + "|gx"] = np64(x), np64(y), np64(xx.grad)
    for name, p in mixer.named_parameters():
        out[k + "|p|" + name] = np64(p)
        out[k + "|g|" + name] = np64(p.grad)

    for cls, wname in [(fdwt.MorletAttention, "freq_weight"),
                       (fdwt.MorletChannelMixAttention, "freq_to_channel")]:
        torch.manual_seed(5)
        m = cls(num_channels=3, hidden_dim=64, temperature=0.5).double()
        x = torch.randn(1, 2, 3, 5, 64, dtype=torch.float64)
        xx = x.clone().requires_grad_()
        y = m(xx)
        y.square().sum().backward()
        k = cls.__name__
        out[k + "|x"], out[k + "|y"], out[k + "|gx"] = np64(x), np64(y), np64(xx.grad)
        for name, p in m.named_parameters():
            out[k + "|p|" + name] = np64(p)
            out[k + "|g|" + name] = np64(p.grad)

    # large amplitudes and a small temperature: the online softmax must stay finite
    torch.manual_seed(6)
    m = fdwt.MorletAttention(num_channels=2, hidden_dim=100, temperature=0.01).double()
    x = 1e3 * torch.randn(1, 1, 2, 4, 100, dtype=torch.float64)
    out["attn_large|x"] = np64(x)
    out["attn_large|y"] = np64(m(x))
    for name, p in m.named_parameters():
        out["attn_large|p|" + name] = np64(p)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference_src)
    import fdwt  # the reference package

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    for name, fn in [("dwt_single", dwt_single), ("dwt_multi", dwt_multi), ("cwt", cwt_cases),
                     ("layers", layer_cases)]:
        out = {}
        fn(fdwt, out)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **out)
        print(f"{path}: {len(out)} arrays, {os.path.getsize(path) / 1e3:.0f} kB")


if __name__ == "__main__":
    main()
