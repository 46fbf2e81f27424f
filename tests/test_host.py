"""Host-side logic that needs no GPU: filter banks, API validation (the reference's exception
types), the no-CPU-fallback rule, and the C ABI library (loads, exports every declared symbol,
rejects bad arguments with a status code before touching a device)."""

import ctypes
import math
import os
import re

import numpy as np
import pytest
import torch

import pytorch_morlet_fdwt_b200 as F
from pytorch_morlet_fdwt_b200 import _build, _lib
from pytorch_morlet_fdwt_b200.wavelets import daubechies_scaling_filter

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fdwt_b200.h")


@pytest.fixture(scope="module")
def lib():
    _build.build()  # incremental: a no-op when the library is up to date
    return _lib.load()


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fdwt_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert len(names) >= 7
    for name in names:
        assert hasattr(lib, name), name
    assert lib.fdwt_version() >= 100
    assert lib.fdwt_status_string(0) == b"ok"


def test_bad_arguments_return_status_without_a_device(lib):
    c = (ctypes.c_int64 * 1)(4)
    outs = (ctypes.c_void_p * 2)(1, 1)
    h = (ctypes.c_double * 2)(0.5, 0.5)
    # odd filter length, negative rows, bad mode, bad dtype
    assert lib.fdwt_dwt_analysis(0, 1, 1, 8, 1, c, None, outs, h, h, 3, 0, 1, None, 0, None) == 1
    assert lib.fdwt_dwt_analysis(0, -1, 1, 8, 1, c, None, outs, h, h, 2, 0, 1, None, 0, None) == 1
    assert lib.fdwt_dwt_analysis(0, 1, 1, 8, 1, c, None, outs, h, h, 2, 9, 1, None, 0, None) == 1
    assert lib.fdwt_dwt_synthesis(0, 1, 1, outs, 7, c, c, 1, h, h, 2, 0, 1, None, 0, None) == 1
    assert lib.fdwt_dwt_analysis(0, 1, 1, 8, 1, c, None, outs, h, h, 66, 0, 1, None, 0, None) == 2
    with pytest.raises(RuntimeError, match="invalid argument"):
        _lib.check(1, "probe")


def test_no_cpu_fallback():
    x = torch.randn(2, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        F.dwt(x, "db2")
    with pytest.raises(RuntimeError, match="CUDA"):
        F.wavedec(x, "db2", level=2)


def test_validation_errors_match_reference():
    x = torch.randn(2, 64)
    with pytest.raises(ValueError):
        F.dwt(x, "morl")
    with pytest.raises(ValueError):
        F.dwt(x, "db2", mode="smooth")
    with pytest.raises(TypeError):
        F.dwt(torch.arange(8), "db2")
    with pytest.raises(ValueError):
        F.idwt(None, None)
    with pytest.raises(ValueError):
        F.idwt(torch.zeros(3), torch.zeros(4))
    with pytest.raises(ValueError):
        F.idwt(torch.zeros(2), torch.zeros(2), "db4")  # 2*2 - 8 + 2 <= 0
    with pytest.raises(ValueError):
        F.wavedec(x, "db2", level=-1)
    with pytest.raises(ValueError):
        F.waverec([])
    with pytest.raises(ValueError):
        F.get_filter_bank(([1.0], [1.0], [1.0]))


def test_daubechies_generator():
    # db2 closed form
    s3 = math.sqrt(3.0)
    ref = np.array([1 + s3, 3 + s3, 3 - s3, 1 - s3]) / (4 * math.sqrt(2.0))
    np.testing.assert_allclose(daubechies_scaling_filter(2), ref, atol=1e-15)
    for order in range(1, 11):
        h = daubechies_scaling_filter(order)
        L = len(h)
        assert L == 2 * order
        assert abs(h.sum() - math.sqrt(2.0)) < 1e-13
        for m in range(order):  # orthonormal to even shifts
            v = sum(h[k] * h[k + 2 * m] for k in range(L - 2 * m))
            assert abs(v - (1.0 if m == 0 else 0.0)) < 1e-12
        g = np.array([(-1) ** k * h[L - 1 - k] for k in range(L)])
        for p in range(order):  # vanishing moments of the wavelet filter
            assert abs(sum(g[k] * k ** p for k in range(L))) < 1e-7 * max(1, L ** p)


def test_named_banks_follow_pywt_conventions():
    b = F.get_filter_bank("db2")
    assert b.length == 4
    np.testing.assert_allclose(b.dec_lo, b.rec_lo[::-1])
    np.testing.assert_allclose(b.dec_hi, b.rec_hi[::-1])
    np.testing.assert_allclose(b.rec_hi, [(-1) ** k * b.rec_lo[3 - k] for k in range(4)])
    haar = F.get_filter_bank("haar")
    np.testing.assert_allclose(haar.dec_hi, [-2 ** -0.5, 2 ** -0.5])
    odd = F.get_filter_bank(([1.0, 2.0, 3.0], [1.0, 0.0, -1.0], [1.0], [2.0]))
    assert odd.length == 4 and odd.rec_lo == (1.0, 0.0, 0.0, 0.0)


def test_dwt_max_level_and_lengths():
    from pytorch_morlet_fdwt_b200.dwt import dwt_coeff_len
    assert F.dwt_max_level(1000, "db4") == 7
    assert F.dwt_max_level(5, "db4") == 0
    assert dwt_coeff_len(65536, 16, "periodization") == 32768
    assert dwt_coeff_len(65536, 16, "symmetric") == 32775
