"""DWT oracle: every level as an explicit sparse operator (TEST INFRASTRUCTURE ONLY).

Restates the reference's CPU path for the Mallat transform:

* ``mode_period`` / ``normalize_mode`` -- ``fdwt/kernels/dwt.py:34-49``;
* ``ext_index`` -- the boundary-extension index map of ``fdwt/reference.py:15-30``;
* ``analysis_operator`` -- ``(A x)[o] = sum_j h[j] x_ext[2o + off - j]`` as the sparse matrix
  ``A`` (``fdwt/reference.py:33-42``, ``fdwt/kernels/dwt.py:3-6``); duplicate index pairs
  (boundary folds) are summed, so ``A.T`` is exactly the reference's synthesis
  (``fdwt/reference.py:45-49``);
* ``dwt``/``idwt``/``wavedec``/``waverec`` -- the API logic of ``fdwt/dwt.py:97-171``
  (coefficient lengths, ``off``, the idwt crop ``2nc - L + 2``, the waverec trim rule);
* ``wavedec_vjp``/``waverec_vjp`` -- gradients, as the transposed operator chains.

Arrays are ``(rows, n)`` numpy arrays; any float dtype works (the operators take the dtype
of the data), so the same code serves as the fp64 checker and the fp32 CPU baseline.
"""

from __future__ import annotations

from functools import lru_cache

import numpy as np
import scipy.sparse as sp

MODES = {"zero": 0, "periodic": 1, "symmetric": 2, "reflect": 3, "periodization": 4}
ZERO, PERIODIC, SYMMETRIC, REFLECT, PERIODIZATION = range(5)


def mode_period(mode: int, n: int) -> int:
    if mode == PERIODIC:
        return n
    if mode == SYMMETRIC:
        return 2 * n
    if mode == REFLECT:
        return 2 * n - 2
    if mode == PERIODIZATION:
        return n + n % 2
    return 1


def normalize_mode(mode: int, n: int) -> int:
    return PERIODIC if (mode == REFLECT and n == 1) else mode


def ext_index(p: np.ndarray, n: int, mode: int):
    """Map extended positions ``p`` onto ``[0, n)``; returns ``(index, valid)``."""
    mode = normalize_mode(mode, n)
    if mode == ZERO:
        valid = (p >= 0) & (p < n)
        return np.clip(p, 0, max(n - 1, 0)), valid
    P = mode_period(mode, n)
    q = np.mod(p, P)
    if mode == PERIODIC:
        idx = q
    elif mode == SYMMETRIC:
        idx = np.where(q < n, q, P - 1 - q)
    elif mode == REFLECT:
        idx = np.where(q < n, q, P - q)
    else:
        idx = np.minimum(q, n - 1)
    return idx, np.ones(p.shape, dtype=bool)


@lru_cache(maxsize=256)
def _operator(n: int, n_out: int, h: tuple, mode: int, off: int) -> sp.csr_matrix:
    L = len(h)
    o = np.arange(n_out)[:, None]
    j = np.arange(L)[None, :]
    idx, valid = ext_index(2 * o + off - j, n, mode)
    rows = np.broadcast_to(o, idx.shape)[valid]
    vals = np.broadcast_to(np.asarray(h, dtype=np.float64)[None, :], idx.shape)[valid]
    return sp.coo_matrix((vals, (rows, idx[valid])), shape=(n_out, n)).tocsr()


def analysis_operator(n: int, n_out: int, h, mode: int, off: int) -> sp.csr_matrix:
    """Sparse ``(n_out, n)`` matrix of one analysis filter (duplicate folds summed)."""
    return _operator(int(n), int(n_out), tuple(float(v) for v in h), int(mode), int(off))


def _apply(A: sp.csr_matrix, x: np.ndarray) -> np.ndarray:
    A = A.astype(x.dtype, copy=False)
    return np.ascontiguousarray((A @ x.T).T)


def _apply_t(A: sp.csr_matrix, y: np.ndarray) -> np.ndarray:
    A = A.astype(y.dtype, copy=False)
    return np.ascontiguousarray((A.T @ y.T).T)


def dwt_coeff_len(n: int, L: int, mode: str) -> int:
    return (n + 1) // 2 if mode == "periodization" else (n + L - 1) // 2


def dwt_max_level(n: int, L: int) -> int:
    if L < 2 or n < L - 1:
        return 0
    return (n // (L - 1)).bit_length() - 1


def _analysis_cfg(bank, mode: str):
    m = MODES[mode]
    L = len(bank[0])
    off = L // 2 if m == PERIODIZATION else 1
    return m, off, L


def dwt(x: np.ndarray, bank, mode: str):
    """``bank = (dec_lo, dec_hi, rec_lo, rec_hi)`` (even length); returns ``(cA, cD)``."""
    m, off, L = _analysis_cfg(bank, mode)
    n = x.shape[-1]
    n_out = dwt_coeff_len(n, L, mode)
    return _apply(analysis_operator(n, n_out, bank[0], m, off), x), \
        _apply(analysis_operator(n, n_out, bank[1], m, off), x)


def dwt_vjp(x_len: int, ga: np.ndarray, gd: np.ndarray, bank, mode: str) -> np.ndarray:
    m, off, L = _analysis_cfg(bank, mode)
    n_out = ga.shape[-1]
    return _apply_t(analysis_operator(x_len, n_out, bank[0], m, off), ga) + \
        _apply_t(analysis_operator(x_len, n_out, bank[1], m, off), gd)


def _synthesis_cfg(bank, mode: str, nc: int):
    L = len(bank[0])
    if mode == "periodization":
        return PERIODIZATION, L // 2, 2 * nc
    n = 2 * nc - L + 2
    if n <= 0:
        raise ValueError(f"coefficients of length {nc} are too short for a filter of length {L}")
    return ZERO, 1, n


def idwt(a: np.ndarray, d: np.ndarray, bank, mode: str) -> np.ndarray:
    """Transpose of the analysis operator built on the reversed ``rec_*`` filters."""
    nc = a.shape[-1]
    m, off, n = _synthesis_cfg(bank, mode, nc)
    lo, hi = tuple(bank[2][::-1]), tuple(bank[3][::-1])
    return _apply_t(analysis_operator(n, nc, lo, m, off), a) + \
        _apply_t(analysis_operator(n, nc, hi, m, off), d)


def idwt_vjp(gy: np.ndarray, nc: int, bank, mode: str):
    m, off, n = _synthesis_cfg(bank, mode, nc)
    lo, hi = tuple(bank[2][::-1]), tuple(bank[3][::-1])
    return _apply(analysis_operator(n, nc, lo, m, off), gy), \
        _apply(analysis_operator(n, nc, hi, m, off), gy)


def wavedec(x: np.ndarray, bank, mode: str, level=None):
    if level is None:
        level = dwt_max_level(x.shape[-1], len(bank[0]))
    details, a = [], x
    for _ in range(level):
        a, d = dwt(a, bank, mode)
        details.append(d)
    return [a] + details[::-1]


def wavedec_vjp(x_len: int, grads, bank, mode: str) -> np.ndarray:
    """Gradient of ``sum <grads[i], wavedec(x)[i]>`` with respect to ``x``."""
    level = len(grads) - 1
    L = len(bank[0])
    lens = [x_len]
    for _ in range(level):
        lens.append(dwt_coeff_len(lens[-1], L, mode))
    g = grads[0]
    for j in range(level, 0, -1):
        g = dwt_vjp(lens[j - 1], g, grads[level - j + 1], bank, mode)
    return g


def waverec(coeffs, bank, mode: str) -> np.ndarray:
    a = coeffs[0]
    for d in coeffs[1:]:
        if a.shape[-1] == d.shape[-1] + 1:
            a = a[..., :-1]
        a = idwt(a, d, bank, mode)
    return a


def waverec_vjp(coeffs, gy: np.ndarray, bank, mode: str):
    """Gradients of ``<gy, waverec(coeffs)>`` with respect to every coefficient array."""
    lens_a = []
    a_len = coeffs[0].shape[-1]
    for d in coeffs[1:]:
        nc = d.shape[-1]
        lens_a.append((a_len, nc))
        a_len = _synthesis_cfg(bank, mode, nc)[2]
    grads_d = []
    g = gy
    for (la, nc) in reversed(lens_a):
        ga, gd = idwt_vjp(g, nc, bank, mode)
        if la == nc + 1:
            ga = np.concatenate([ga, np.zeros_like(ga[..., :1])], axis=-1)
        grads_d.append(gd)
        g = ga
    return [g] + grads_d[::-1]
