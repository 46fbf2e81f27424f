"""ctypes binding of ``libfdwt_b200.so`` (the C ABI declared in ``include/fdwt_b200.h``).

The library is loaded on first use.  There is no fallback: if the shared library is missing
or the tensors are not on a CUDA device, the call raises.  Status codes other than
``FDWT_OK`` become ``RuntimeError`` with the library's message.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libfdwt_b200.so")

c_i64p = ctypes.POINTER(ctypes.c_int64)
c_dblp = ctypes.POINTER(ctypes.c_double)
c_voidpp = ctypes.POINTER(ctypes.c_void_p)

DTYPES = {torch.float32: 0, torch.float64: 1, torch.float16: 2, torch.bfloat16: 3}

# name -> (restype, argtypes)
SIGNATURES = {
    "fdwt_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "fdwt_last_cuda_error": (ctypes.c_int, []),
    "fdwt_version": (ctypes.c_int, []),
    "fdwt_launch_count": (ctypes.c_ulonglong, []),
    "fdwt_set_shared_memory_fill": (None, [ctypes.c_int, ctypes.c_uint]),
    "fdwt_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "fdwt_set_copy_wait_test": (None, [ctypes.c_uint, ctypes.c_longlong]),
    "fdwt_set_cwt_tile_test": (None, [ctypes.c_int]),
    "fdwt_dwt_analysis_noalloc": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, c_i64p, c_i64p,
        c_voidpp, c_dblp, c_dblp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "fdwt_dwt_analysis": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, c_i64p, c_i64p,
        c_voidpp, c_dblp, c_dblp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
        ctypes.c_size_t, ctypes.c_void_p]),
    "fdwt_dwt_analysis_workspace": (ctypes.c_size_t, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, c_i64p, c_i64p, ctypes.c_int,
        ctypes.c_int, ctypes.c_int]),
    "fdwt_dwt_synthesis": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int, c_voidpp, ctypes.c_int64, c_i64p, c_i64p,
        ctypes.c_void_p, c_dblp, c_dblp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
        ctypes.c_size_t, ctypes.c_void_p]),
    "fdwt_cwt_forward": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "fdwt_mix_forward": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_void_p]),
    "fdwt_specsoftmax_forward": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_double,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "fdwt_cwt_backward_workspace": (ctypes.c_size_t, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int]),
    "fdwt_cwt_backward": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_size_t, ctypes.c_void_p]),
    "fdwt_mix_backward_workspace": (ctypes.c_size_t, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
        ctypes.c_int]),
    "fdwt_mix_backward": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_size_t, ctypes.c_void_p]),
    "fdwt_mix_tokens_forward": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p]),
    "fdwt_mix_tokens_backward_workspace": (ctypes.c_size_t, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_int]),
    "fdwt_mix_tokens_backward": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "fdwt_specsoftmax_backward_workspace": (ctypes.c_size_t, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int,
        ctypes.c_int64, ctypes.c_int]),
    "fdwt_specsoftmax_backward": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_double,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "fdwt_dwt_synthesis_workspace": (ctypes.c_size_t, [
        ctypes.c_int, ctypes.c_int64, ctypes.c_int, ctypes.c_int64, c_i64p, c_i64p, ctypes.c_int,
        ctypes.c_int, ctypes.c_int]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the shared library; raises if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build the sm_100a kernels with "
                        "`python -m pytorch_morlet_fdwt_b200._build` (or __graft_entry__.build())")
                lib = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.restype, fn.argtypes = res, args
                _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        lib = load()
        msg = lib.fdwt_status_string(status).decode()
        if status == 4:
            msg += f" (cudaError {lib.fdwt_last_cuda_error()})"
        raise RuntimeError(f"{what} failed: {msg}")


def require_cuda(*tensors) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "pytorch_morlet_fdwt_b200 computes on CUDA tensors only (sm_100a kernels, no CPU "
                f"fallback); got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPES[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}") from None


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def i64_array(values):
    arr = (ctypes.c_int64 * max(1, len(values)))(*[int(v) for v in values])
    return arr


def f64_array(values):
    return (ctypes.c_double * max(1, len(values)))(*[float(v) for v in values])


def ptr_array(tensors):
    return (ctypes.c_void_p * max(1, len(tensors)))(
        *[None if t is None else t.data_ptr() for t in tensors])


def workspace(nbytes: int, device: torch.device):
    if nbytes == 0:
        return None
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device)


def launch_count() -> int:
    """Kernels launched by libfdwt_b200.so so far in this process."""
    return int(load().fdwt_launch_count())


def device_error() -> int:
    """Read and clear the device-side error word (nonzero: a kernel gave up waiting on an
    asynchronous copy and left its work unfinished)."""
    v = ctypes.c_int(0)
    check(load().fdwt_device_error(ctypes.byref(v)), "fdwt_device_error")
    return int(v.value)


def check_device_error(what: str) -> None:
    """Raise if a kernel gave up waiting on a copy since the last check (synchronises the
    device).  Called after every DWT call while ``config.check_device_errors`` is set."""
    code = device_error()
    if code != 0:
        raise RuntimeError(
            f"{what}: a streaming kernel's bounded wait on an asynchronous copy ran out (device "
            f"error {code}); its outputs are incomplete")


def set_copy_wait_test(extra_tx_bytes: int, tries: int = 0) -> None:
    """Test hook: make the bounded copy wait of global tile 0 run out (see
    fdwt_set_copy_wait_test); ``(0, 0)`` restores the defaults."""
    load().fdwt_set_copy_wait_test(int(extra_tx_bytes), int(tries))


def set_cwt_tile_test(t_len: int) -> None:
    """Test hook: run every Morlet call on time tiles of ``t_len`` positions (0: automatic)."""
    load().fdwt_set_cwt_tile_test(int(t_len))


def set_shared_memory_fill(enable: bool, word: int = 0) -> None:
    """Test hook: while enabled, every kernel of the library is preceded by one that sets all
    shared memory to the 32-bit pattern `word` (see fdwt_set_shared_memory_fill)."""
    load().fdwt_set_shared_memory_fill(1 if enable else 0, word & 0xFFFFFFFF)
