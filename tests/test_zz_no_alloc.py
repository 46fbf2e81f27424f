"""fdwt_dwt_analysis_noalloc, the allocation-free analysis entry point, called through the C ABI.

Its output must match fdwt_dwt_analysis (the entry point that takes a caller workspace) on
rows long enough that the levels are split over several launches, which hand the approximation
over through the library's static scratch array.  Two calls in a row on different data check
that nothing from the first call leaks into the second.  This file is collected last so that a
run stopping at the first failure has already run every other test.
"""

import ctypes

import pytest
import torch

import pytorch_morlet_fdwt_b200 as F
from pytorch_morlet_fdwt_b200 import _lib
from pytorch_morlet_fdwt_b200.dwt import MODES, _analysis_spec

pytestmark = pytest.mark.gpu
DEV = "cuda"
SCRATCH_LIMIT = 16 << 20
FDWT_ERR_SCRATCH_LIMIT = 5


def _noalloc():
    lib = _lib.load()
    fn = lib.fdwt_dwt_analysis_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                   _lib.c_i64p, _lib.c_i64p, _lib.c_voidpp, _lib.c_dblp, _lib.c_dblp,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return lib, fn


def _need(dtype, rows, n, bank, mode, level):
    """Workspace bytes fdwt_dwt_analysis asks for (0 when one launch holds every level)."""
    spec = _analysis_spec(bank, MODES[mode], n, level, mode)
    return _lib.load().fdwt_dwt_analysis_workspace(
        _lib.dtype_code(dtype), rows, n, level, _lib.i64_array(spec.coef_len),
        _lib.i64_array(spec.pad), len(spec.h0), spec.mode, spec.off)


def _multi_launch_length(dtype, rows, bank, mode, level):
    """Shortest power-of-two row length whose levels need several launches on this GPU."""
    for log_n in range(14, 23):
        if _need(dtype, rows, 1 << log_n, bank, mode, level) > 0:
            return 1 << log_n
    raise AssertionError("no row length up to 2^22 splits into several launches")


def _call(x, bank, mode, level):
    """Run the no-alloc entry point on the rows of x; returns (status, [cA, cD_J, ..., cD_1])."""
    lib, fn = _noalloc()
    spec = _analysis_spec(bank, MODES[mode], x.shape[-1], level, mode)
    R = x.shape[0]
    outs = [torch.empty((R, spec.approx_len), device=x.device, dtype=x.dtype)]
    outs += [torch.empty((R, c), device=x.device, dtype=x.dtype) for c in reversed(spec.coef_len)]
    need = lib.fdwt_dwt_analysis_workspace(
        _lib.dtype_code(x.dtype), R, spec.n, level, _lib.i64_array(spec.coef_len),
        _lib.i64_array(spec.pad), len(spec.h0), spec.mode, spec.off)
    st = fn(_lib.dtype_code(x.dtype), R, x.data_ptr(), spec.n, level,
            _lib.i64_array(spec.coef_len), _lib.i64_array(spec.pad), _lib.ptr_array(outs),
            _lib.f64_array(spec.h0), _lib.f64_array(spec.h1), len(spec.h0), spec.mode, spec.off,
            _lib.stream_of(x.device))
    return st, need, outs


def _close(a, b, tol):
    scale = max(float(b.abs().max()), 1.0)
    err = float((a - b).abs().max())
    assert err <= tol * scale, f"max err {err:.3e} > {tol:.1e} x {scale:.3e}"


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-12), (torch.float32, 1e-5)])
@pytest.mark.parametrize("mode", ["symmetric", "periodization"])
def test_noalloc_matches_workspace_entry_two_calls(dtype, tol, mode):
    torch.manual_seed(11)
    bank = F.get_filter_bank("db4")
    rows, level = 2, 10
    n = _multi_launch_length(dtype, rows, bank, mode, level)
    for call in range(2):
        x = torch.randn(rows, n, dtype=dtype, device=DEV) * (call + 1)
        before = _lib.launch_count()
        st, need, outs = _call(x, bank, mode, level)
        _lib.check(st, "fdwt_dwt_analysis_noalloc")
        assert _lib.launch_count() - before >= 2  # several launches, so the scratch is used
        assert 0 < need <= SCRATCH_LIMIT
        ref = F.wavedec(x, bank, mode, level)  # fdwt_dwt_analysis with a torch workspace
        assert len(ref) == len(outs)
        for o, r in zip(outs, ref):
            assert o.shape == r.shape
            _close(o, r, tol)


def test_noalloc_rejects_sizes_beyond_the_scratch():
    bank = F.get_filter_bank("db4")
    n = _multi_launch_length(torch.float32, 1, bank, "symmetric", 10)
    # the workspace grows with the rows up to a per-region rounding to 256 bytes
    rows = SCRATCH_LIMIT // _need(torch.float32, 1, n, bank, "symmetric", 10) + 1
    while _need(torch.float32, rows, n, bank, "symmetric", 10) <= SCRATCH_LIMIT:
        rows += 1
    assert rows * n * 4 <= 1 << 31
    x = torch.zeros(rows, n, dtype=torch.float32, device=DEV)
    before = _lib.launch_count()
    st, need, _ = _call(x, bank, "symmetric", 10)
    assert need > SCRATCH_LIMIT
    assert st == FDWT_ERR_SCRATCH_LIMIT
    assert b"no-allocation" in _lib.load().fdwt_status_string(st)
    assert _lib.launch_count() == before


@pytest.mark.parametrize("mode", ["symmetric", "periodization"])
def test_noalloc_misaligned_rows_match(mode):
    """Rows that start 4 bytes past a 16-byte boundary (a contiguous view at an odd storage
    offset) cannot stream; the call takes the cluster plan, whose workspace the query and the
    static array must cover as well."""
    torch.manual_seed(12)
    bank = F.get_filter_bank("db4")
    rows, level = 2, 10
    n = _multi_launch_length(torch.float32, rows, bank, mode, level)
    for call in range(2):
        flat = torch.randn(1 + rows * n, dtype=torch.float32, device=DEV) * (call + 1)
        x = flat[1:].view(rows, n)
        assert x.data_ptr() % 16 != 0
        st, need, outs = _call(x, bank, mode, level)
        _lib.check(st, "fdwt_dwt_analysis_noalloc")
        assert 0 < need <= SCRATCH_LIMIT
        ref = F.wavedec(x.clone(), bank, mode, level)  # aligned copy
        for o, r in zip(outs, ref):
            _close(o, r, 1e-5)
