"""The bounded copy waits of the streaming DWT kernels, made to run out on purpose.

``fdwt_set_copy_wait_test`` makes the kernels expect 16 bytes more than they copy for global
tile 0 (a wait for bytes that never come, with every issued copy still landing) and shortens
the poll limit of the main waits.  The kernel must then store 1 in the device error word, wait
for its copies still in flight and return, leaving the context usable; ``fdwt_device_error``
reads and clears the word, and with ``config.check_device_errors`` the DWT call itself raises.
Nothing here faults: the only thing changed is the byte count a wait expects.
"""

import numpy as np
import pytest
import torch

import pytorch_morlet_fdwt_b200 as F
from pytorch_morlet_fdwt_b200 import _lib, config
from oracle import dwt_oracle as D

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run(case, x, c, bank):
    if case.startswith("ana"):
        return F.wavedec(x, bank, "periodization", 1 if case == "ana1" else 2)
    return F.waverec(c, bank, "periodization")


@pytest.mark.parametrize("case", ["ana1", "ana2", "syn1", "syn2"])
def test_wait_that_runs_out_sets_the_error_word(case):
    torch.manual_seed(5)
    bank = F.get_filter_bank("db8")
    x = torch.randn(8, 65536, device=DEV)
    level = 1 if case.endswith("1") else 2
    c = F.wavedec(x, bank, "periodization", level)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    _lib.set_copy_wait_test(16, 1 << 12)
    try:
        _run(case, x, c, bank)
        torch.cuda.synchronize()
    finally:
        _lib.set_copy_wait_test(0, 0)
    assert _lib.device_error() == 1  # a streaming kernel gave up on tile 0 and returned
    assert _lib.device_error() == 0  # reading clears the word
    # the context is still usable and a normal call is right again
    b = (bank.dec_lo, bank.dec_hi, bank.rec_lo, bank.rec_hi)
    xr = x.double().cpu().numpy()
    ref = D.wavedec(xr, b, "periodization", level)
    if case.startswith("ana"):
        got = _run(case, x, c, bank)
        for g, r in zip(got, ref):
            err = np.abs(g.double().cpu().numpy() - r).max()
            assert err <= 1e-5 * np.abs(r).max()
    else:
        y = _run(case, x, c, bank).double().cpu().numpy()
        assert np.abs(y - xr).max() <= 1e-5 * np.abs(xr).max()  # perfect reconstruction
    assert _lib.device_error() == 0


def test_opt_in_check_raises():
    bank = F.get_filter_bank("db8")
    x = torch.randn(4, 65536, device=DEV)
    config.check_device_errors = True
    try:
        F.wavedec(x, bank, "periodization", 2)  # no timeout: no error
        _lib.set_copy_wait_test(16, 1 << 12)
        try:
            with pytest.raises(RuntimeError, match="bounded wait"):
                F.wavedec(x, bank, "periodization", 2)
        finally:
            _lib.set_copy_wait_test(0, 0)
        F.wavedec(x, bank, "periodization", 2)
    finally:
        config.check_device_errors = False
    assert _lib.device_error() == 0
