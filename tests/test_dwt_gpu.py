"""DWT parity on the GPU: sm_100a kernels (through the C ABI) vs the golden fixtures and the
CPU oracle, plus size-independent properties at the benchmark sizes.

Tolerances: fp64 1e-12 x max|ref| (the reference's pywt tolerance, tests/test_dwt.py:32), fp32
1e-5 relative to max|ref| (the north-star bound for DWT coefficients), fp16 1e-2, bf16 6e-2
(the reference's low-precision test, tests/test_dwt.py:82).
"""

import numpy as np
import pytest
import torch
from torch.autograd import gradcheck, gradgradcheck

import pytorch_morlet_fdwt_b200 as F
from pytorch_morlet_fdwt_b200 import _lib
from oracle import dwt_oracle as D
from tests.golden_data import bank_from_golden, golden

pytestmark = pytest.mark.gpu
MODES = ["zero", "periodic", "symmetric", "reflect", "periodization"]
DEV = "cuda"


def close(a, b, tol, floor=0.0):
    """max|a - b| <= tol * max(max|b|, floor): relative to the reference's magnitude, with an
    absolute floor for the O(1)-scaled golden cases (pywt's own tests use atol=1e-12)."""
    a = a.detach().double().cpu().numpy() if torch.is_tensor(a) else np.asarray(a)
    b = b.detach().double().cpu().numpy() if torch.is_tensor(b) else np.asarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    scale = max(floor, 1e-300, float(np.abs(b).max()) if b.size else 1.0)
    err = float(np.abs(a - b).max()) if b.size else 0.0
    assert err <= tol * scale, f"max err {err:.3e} > {tol:.1e} x {scale:.3e}"


def gpu(a, dtype=torch.float64):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


@pytest.mark.parametrize("bname", ["haar", "db2", "db4", "rand5"])
@pytest.mark.parametrize("mode", MODES)
def test_single_level_vs_golden(bname, mode):
    g = golden("dwt_single")
    bank = F.get_filter_bank(bank_from_golden(bname))
    for n in [1, 2, 3, 7, 16, 33, 100]:
        key = f"{bname}|{mode}|{n}"
        x = gpu(g[key + "|x"])
        a, d = F.dwt(x, bank, mode)
        close(a, g[key + "|a"], 1e-12, 1.0)
        close(d, g[key + "|d"], 1e-12, 1.0)
        xg = x.clone().requires_grad_()
        a2, d2 = F.dwt(xg, bank, mode)
        (a2.square().sum() + 3.0 * d2.square().sum()).backward()
        close(xg.grad, g[key + "|gx"], 1e-12, 1.0)
        if key + "|y" in g:
            close(F.idwt(a, d, bank, mode), g[key + "|y"], 1e-12, 1.0)
            ag, dg = a.clone().requires_grad_(), d.clone().requires_grad_()
            F.idwt(ag, dg, bank, mode).square().sum().backward()
            close(ag.grad, g[key + "|ga"], 1e-12, 1.0)
            close(dg.grad, g[key + "|gd"], 1e-12, 1.0)
        else:
            with pytest.raises(ValueError):
                F.idwt(a, d, bank, mode)


def _multi_keys():
    g = golden("dwt_multi")
    return sorted({k.rsplit("|", 1)[0] for k in g.files if k.endswith("|x")})


@pytest.mark.parametrize("key", _multi_keys())
def test_multilevel_vs_golden(key):
    g = golden("dwt_multi")
    bname, mode, n = key.split("|")
    bank = F.get_filter_bank(bank_from_golden(bname))
    level = int(g[key + "|level"])
    x = gpu(g[key + "|x"]).requires_grad_()
    coeffs = F.wavedec(x, bank, mode, level)
    assert len(coeffs) == level + 1
    for i, c in enumerate(coeffs):
        close(c, g[key + f"|c{i}"], 1e-12, 1.0)
    sum((c.square() * (1.0 + i)).sum() for i, c in enumerate(coeffs)).backward()
    close(x.grad, g[key + "|gx"], 1e-12, 1.0)
    cs = [gpu(g[key + f"|c{i}"]).requires_grad_() for i in range(level + 1)]
    y = F.waverec(cs, bank, mode)
    close(y, g[key + "|y"], 1e-12, 1.0)
    y.square().sum().backward()
    for i, c in enumerate(cs):
        close(c.grad, g[key + f"|gc{i}"], 1e-12, 1.0)


@pytest.mark.parametrize("mode", MODES)
def test_gradcheck_and_double_backward(mode):
    torch.manual_seed(0)
    for wname in ["haar", "db3"]:
        bank = F.get_filter_bank(wname)
        for n in [1, 2, 5, 8, 13, 40]:
            x = torch.randn(2, n, dtype=torch.float64, device=DEV, requires_grad=True)
            assert gradcheck(lambda t: F.dwt(t, bank, mode), (x,))
            assert gradgradcheck(lambda t: F.dwt(t, bank, mode), (x,))
            a, d = (t.detach().requires_grad_() for t in F.dwt(x, bank, mode))
            if mode == "periodization" or 2 * a.shape[-1] - bank.length + 2 > 0:
                assert gradcheck(lambda p, q: F.idwt(p, q, bank, mode), (a, d))
        x = torch.randn(3, 37, dtype=torch.float64, device=DEV, requires_grad=True)
        assert gradgradcheck(lambda t: F.wavedec(t, bank, mode, 3), (x,))


def test_cfg1_wavedec_waverec_fp32():
    """db4 symmetric level 5 on (32, 64, 2500) fp32, forward + backward of sum c^2."""
    torch.manual_seed(0)
    bank = F.get_filter_bank("db4")
    tb = (bank.dec_lo, bank.dec_hi, bank.rec_lo, bank.rec_hi)
    x = torch.randn(32, 64, 2500, device=DEV).requires_grad_()
    coeffs = F.wavedec(x, "db4", "symmetric", 5)
    x64 = x.detach().double().cpu().numpy().reshape(-1, 2500)
    ref = D.wavedec(x64, tb, "symmetric", 5)
    for c, r in zip(coeffs, ref):
        close(c.reshape(-1, c.shape[-1]), r, 1e-5)
    sum(c.square().sum() for c in coeffs).backward()
    gref = D.wavedec_vjp(2500, [2 * r for r in ref], tb, "symmetric")
    close(x.grad.reshape(-1, 2500), gref, 1e-5)
    y = F.waverec([c.detach() for c in coeffs], "db4", "symmetric")
    close(y.reshape(-1, y.shape[-1]), D.waverec(ref, tb, "symmetric"), 1e-5)
    close(y[..., :2500], x.detach(), 1e-5)


@pytest.mark.parametrize("mode", MODES)
def test_cfg2_long_signal_fp32(mode):
    """db8 level 8 on (16, 128, 65536) fp32 -- every mode.  Sampled rows against the
    oracle, every row through size-independent properties (adjointness, reconstruction)."""
    torch.manual_seed(1)
    bank = F.get_filter_bank("db8")
    tb = (bank.dec_lo, bank.dec_hi, bank.rec_lo, bank.rec_hi)
    x = torch.randn(16, 128, 65536, device=DEV)
    coeffs = F.wavedec(x, bank, mode, 8)
    rows = [0, 1, 777, 2047]
    xr = x.reshape(-1, 65536)[rows].double().cpu().numpy()
    ref = D.wavedec(xr, tb, mode, 8)
    for c, r in zip(coeffs, ref):
        close(c.reshape(-1, c.shape[-1])[rows], r, 1e-5)
    # adjointness <A x, g> == <x, A^T g> on every row (fp64 accumulation of fp32 kernels)
    gs = [torch.randn_like(c) for c in coeffs]
    xx = x.clone().requires_grad_()
    cs = F.wavedec(xx, bank, mode, 8)
    torch.autograd.backward(cs, gs)
    lhs = sum((c.double() * g.double()).sum() for c, g in zip(coeffs, gs))
    rhs = (x.double() * xx.grad.double()).sum()
    assert abs(float(lhs - rhs)) <= 1e-5 * float(lhs.abs() + rhs.abs())
    gref = D.wavedec_vjp(65536, [g.reshape(-1, g.shape[-1])[rows].double().cpu().numpy()
                                 for g in gs], tb, mode)
    close(xx.grad.reshape(-1, 65536)[rows], gref, 1e-5)
    # reconstruction and the waverec backward
    cs2 = [c.detach().requires_grad_() for c in coeffs]
    y = F.waverec(cs2, bank, mode)
    close(y.reshape(-1, y.shape[-1])[rows], D.waverec(ref, tb, mode), 1e-5)
    close(y[..., :65536], x, 1e-5)
    gy = torch.randn_like(y)
    y.backward(gy)
    gr = D.waverec_vjp(ref, gy.reshape(-1, y.shape[-1])[rows].double().cpu().numpy(), tb, mode)
    for c, r in zip(cs2, gr):
        close(c.grad.reshape(-1, c.shape[-1])[rows], r, 1e-5)


def test_long_rows_fp64_multi_segment():
    """fp64 rows of 65536 do not fit one launch's shared memory: the levels are split into
    launches that hand the approximation over through the workspace."""
    torch.manual_seed(2)
    bank = F.get_filter_bank("db4")
    tb = (bank.dec_lo, bank.dec_hi, bank.rec_lo, bank.rec_hi)
    for mode in ["symmetric", "periodization"]:
        x = torch.randn(3, 65536, dtype=torch.float64, device=DEV)
        coeffs = F.wavedec(x, bank, mode, 10)
        ref = D.wavedec(x.cpu().numpy(), tb, mode, 10)
        for c, r in zip(coeffs, ref):
            close(c, r, 1e-12, 1.0)
        y = F.waverec(coeffs, bank, mode)
        close(y, D.waverec(ref, tb, mode), 1e-12, 1.0)
        xx = x.clone().requires_grad_()
        sum(c.square().sum() for c in F.wavedec(xx, bank, mode, 10)).backward()
        close(xx.grad, D.wavedec_vjp(65536, [2 * r for r in ref], tb, mode), 1e-12, 1.0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_low_precision_dtypes(dtype):
    torch.manual_seed(0)
    x = torch.randn(4, 1000, device=DEV)
    ref = F.wavedec(x.double(), "db4", level=4)
    out = F.wavedec(x.to(dtype), "db4", level=4)
    tol = {torch.float32: 1e-5, torch.float16: 1e-2, torch.bfloat16: 6e-2}[dtype]
    for o, r in zip(out, ref):
        assert o.dtype == dtype
        torch.testing.assert_close(o.double(), r, atol=tol * r.abs().max().item(), rtol=0)
    y = F.waverec(out, "db4")
    assert y.dtype == dtype


def test_gpu_matches_oracle_large_batch():
    torch.manual_seed(0)
    bank = F.get_filter_bank("db4")
    tb = (bank.dec_lo, bank.dec_hi, bank.rec_lo, bank.rec_hi)
    x = torch.randn(5, 7, 2049)
    xg = x.cuda().requires_grad_()
    outs = F.wavedec(xg, bank, "reflect")
    ref = D.wavedec(x.double().numpy().reshape(-1, 2049), tb, "reflect")
    for a, b in zip(outs, ref):
        close(a.reshape(-1, a.shape[-1]), b, 1e-5)
    sum((c * c).sum() for c in outs).backward()
    close(xg.grad.reshape(-1, 2049), D.wavedec_vjp(2049, [2 * r for r in ref], tb, "reflect"), 1e-4)


def test_modules_and_errors():
    x = torch.randn(2, 128, device=DEV)
    m, im = F.DWT1D("db2", level=3), F.IDWT1D("db2")
    torch.testing.assert_close(im(m(x))[..., :128], x, atol=1e-5, rtol=1e-5)
    with pytest.raises(ValueError):
        F.dwt(x, "morl")
    with pytest.raises(ValueError):
        F.dwt(x, "db2", mode="smooth")
    b = F.get_filter_bank("db2")
    custom = F.get_filter_bank((b.dec_lo, b.dec_hi, b.rec_lo, b.rec_hi))
    torch.testing.assert_close(F.dwt(x, custom)[0], F.dwt(x, "db2")[0])
    assert F.dwt_max_level(1000, "db4") == D.dwt_max_level(1000, 8) == 7
    assert F.wavedec(x, "db2", level=0)[0] is x


def test_empty_batch_and_noncontiguous():
    x = torch.randn(0, 3, 50, device=DEV)
    a, d = F.dwt(x, "db2")
    assert a.shape == (0, 3, 26) and d.shape == (0, 3, 26)
    base = torch.randn(40, 6, device=DEV, dtype=torch.float64)
    xt = base.t()  # (6, 40), non-contiguous rows
    bank = F.get_filter_bank("db2")
    tb = (bank.dec_lo, bank.dec_hi, bank.rec_lo, bank.rec_hi)
    for c, r in zip(F.wavedec(xt, bank, "symmetric", 2),
                    D.wavedec(xt.cpu().numpy(), tb, "symmetric", 2)):
        close(c, r, 1e-12, 1.0)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.float64, 1e-12)])
@pytest.mark.parametrize("wname,mode,nc", [("db8", "periodization", 32768), ("db4", "periodization", 16384),
                                           ("haar", "periodization", 16384), ("db10", "periodization", 12288),
                                           ("db12", "periodization", 12288), ("db3", "zero", 8196),
                                           ("db4", "reflect", 8192), ("db20", "periodization", 16384)])
def test_one_level_synthesis_long_rows(wname, mode, nc, dtype, tol):
    """One-level syntheses of long rows: interior tiles on the streaming kernel (bulk copies
    through an mbarrier ring; filters up to 24 taps, rows whose lengths are multiples of 16
    bytes), the tiles near the row ends -- and every tile of db20 -- on the tile kernel.  Also
    the same level as the last stage of a deeper waverec, and the device error word stays 0."""
    torch.manual_seed(11)
    bank = F.get_filter_bank(wname)
    tb = (bank.dec_lo, bank.dec_hi, bank.rec_lo, bank.rec_hi)
    a = torch.randn(5, nc, dtype=dtype, device=DEV)
    d = torch.randn(5, nc, dtype=dtype, device=DEV)
    y = F.idwt(a, d, bank, mode)
    close(y, D.idwt(a.double().cpu().numpy(), d.double().cpu().numpy(), tb, mode), tol)
    ag, dg = a.clone().requires_grad_(), d.clone().requires_grad_()
    gy = torch.randn_like(y)
    (F.idwt(ag, dg, bank, mode) * gy).sum().backward()
    ga, gd = D.idwt_vjp(gy.double().cpu().numpy(), nc, tb, mode)
    close(ag.grad, ga, tol)
    close(dg.grad, gd, tol)
    x = torch.randn(3, y.shape[-1], dtype=dtype, device=DEV)
    for levels in (2, 3):  # two levels: one fused pass where the pair fuses
        coeffs = F.wavedec(x, bank, mode, levels)
        ref = D.wavedec(x.double().cpu().numpy(), tb, mode, levels)
        close(F.waverec(coeffs, bank, mode), D.waverec(ref, tb, mode), tol)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.float64, 1e-12)])
@pytest.mark.parametrize("wname,mode,n", [("db8", "periodization", 65536), ("db8", "symmetric", 16384),
                                          ("db4", "reflect", 12288), ("haar", "zero", 4096),
                                          ("db10", "periodic", 8192), ("db12", "periodization", 6148),
                                          ("db7", "symmetric", 4104), ("db20", "symmetric", 8192)])
def test_one_level_analysis_long_rows(wname, mode, n, dtype, tol):
    """One-level analyses of rows of a multiple of 16 bytes: every tile on the streaming kernel
    (bulk copies through an mbarrier ring, the extended positions past the row ends gathered
    through the boundary map; filters up to 24 taps -- db20 stays on the cluster kernel), as a
    single level and as the finest levels of a deeper wavedec, forward and backward (the
    backward of waverec is an analysis whose approximation carries a trailing zero)."""
    torch.manual_seed(12)
    bank = F.get_filter_bank(wname)
    tb = (bank.dec_lo, bank.dec_hi, bank.rec_lo, bank.rec_hi)
    x = torch.randn(5, n, dtype=dtype, device=DEV)
    a, d = F.dwt(x, bank, mode)
    ra, rd = D.dwt(x.double().cpu().numpy(), tb, mode)
    close(a, ra, tol)
    close(d, rd, tol)
    coeffs = F.wavedec(x, bank, mode, 4)
    ref = D.wavedec(x.double().cpu().numpy(), tb, mode, 4)
    for c, r in zip(coeffs, ref):
        close(c, r, tol)
    cg = [c.clone().requires_grad_() for c in coeffs]
    y = F.waverec(cg, bank, mode)
    gy = torch.randn_like(y)
    (y * gy).sum().backward()
    for c, r in zip(cg, D.waverec_vjp(ref, gy.double().cpu().numpy(), tb, mode)):
        close(c.grad, r, tol)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


@pytest.mark.parametrize("mode", MODES)
def test_per_level_nodes_apply_vs_golden(mode):
    """The reference's per-level autograd nodes, called through ``apply`` with the reference's
    signatures (``fdwt/dwt.py:36-82``): ``_Analysis.apply(x, h0, h1, mode, off, n_out)`` gives
    pywt's dwt, ``_Synthesis.apply(a, d, rec_lo[::-1], rec_hi[::-1], mode, off, n)`` pywt's idwt
    (zero mode, or periodization), and their gradients match the fixtures."""
    from pytorch_morlet_fdwt_b200.dwt import MODES as IDS, _Analysis, _Synthesis, dwt_coeff_len
    g = golden("dwt_single")
    for bname in ["haar", "db4", "rand5"]:
        bank = F.get_filter_bank(bank_from_golden(bname))
        L = bank.length
        h0, h1 = gpu(bank.dec_lo), gpu(bank.dec_hi)
        r0, r1 = gpu(bank.rec_lo[::-1]), gpu(bank.rec_hi[::-1])
        off = L // 2 if mode == "periodization" else 1
        for n in [7, 16, 33, 100]:
            key = f"{bname}|{mode}|{n}"
            x = gpu(g[key + "|x"]).requires_grad_()
            n_out = dwt_coeff_len(n, L, mode)
            a, d = _Analysis.apply(x, h0, h1, IDS[mode], off, n_out)
            close(a, g[key + "|a"], 1e-12, 1.0)
            close(d, g[key + "|d"], 1e-12, 1.0)
            (a.square().sum() + 3.0 * d.square().sum()).backward()
            close(x.grad, g[key + "|gx"], 1e-12, 1.0)
            if key + "|y" not in g:
                continue
            if mode == "periodization":
                sm, soff, ny = IDS["periodization"], L // 2, 2 * n_out
            else:
                sm, soff, ny = IDS["zero"], 1, 2 * n_out - L + 2
            ag = a.detach().clone().requires_grad_()
            dg = d.detach().clone().requires_grad_()
            y = _Synthesis.apply(ag, dg, r0, r1, sm, soff, ny)
            close(y, g[key + "|y"], 1e-12, 1.0)
            y.square().sum().backward()
            close(ag.grad, g[key + "|ga"], 1e-12, 1.0)
            close(dg.grad, g[key + "|gd"], 1e-12, 1.0)


@pytest.mark.parametrize("mode", ["symmetric", "periodization"])
def test_misaligned_rows_on_a_multi_launch_length(mode):
    """A contiguous view at an odd storage offset (rows not 16-byte aligned) does not stream and
    falls back to the cluster plan at run time; the workspace the query returned covers it."""
    torch.manual_seed(21)
    bank = F.get_filter_bank("db8")
    rows, n = 16, 1 << 18
    flat = torch.randn(1 + rows * n, device=DEV)
    x = flat[1:].view(rows, n)
    assert x.data_ptr() % 16 != 0
    got = F.wavedec(x, bank, mode, 8)
    ref = F.wavedec(x.clone(), bank, mode, 8)
    for g, r in zip(got, ref):
        close(g, r, 1e-5)
    y = F.waverec(got, bank, mode)
    close(y[..., :n], x, 1e-5)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.float64, 1e-12)])
@pytest.mark.parametrize("mode", ["zero", "periodic", "symmetric", "reflect"])
@pytest.mark.parametrize("wname", ["haar", "db3", "db8", "db12"])
def test_padded_handovers_between_streaming_stages(wname, mode, dtype, tol):
    """Coefficient lengths are odd in every mode but periodization, so the approximation one
    streaming pass hands to the next is stored in the workspace with its rows rounded up to 16
    bytes; the next pass bulk-copies up to the last 16-byte boundary of each row and gathers the
    ragged end.  Every row of every level against the oracle, at lengths whose intermediate
    approximations take every residue mod 16 bytes, then the round trip."""
    torch.manual_seed(31)
    bank = F.get_filter_bank(wname)
    tb = (bank.dec_lo, bank.dec_hi, bank.rec_lo, bank.rec_hi)
    for n in (16384, 20004, 24584):
        x = torch.randn(6, n, device=DEV, dtype=dtype)
        level = min(7, F.dwt_max_level(n, wname))
        got = F.wavedec(x, bank, mode, level)
        ref = D.wavedec(x.double().cpu().numpy(), tb, mode, level)
        for g, r in zip(got, ref):
            close(g, r, tol)
        y = F.waverec(got, bank, mode)
        close(y[..., :n], x, tol)
