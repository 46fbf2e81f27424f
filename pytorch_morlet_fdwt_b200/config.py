"""Global switches (``allow_tf32`` / ``allow_bf16`` have the names and defaults of the
reference's ``fdwt/config.py:17-18``).

``allow_tf32`` and ``allow_bf16`` are accepted for drop-in compatibility.  In the reference
they let the Triton dots take TF32 / bf16 operands (``fdwt/kernels/conv.py:332-338``) for speed.
The sm_100a kernels compute every filter-bank contraction with fp32 FMAs for fp32/fp16/bf16
inputs and fp64 FMAs for fp64 inputs whatever they say: on B200 a TF32 tensor-core filter stage
(warp-level ``mma.sync``) measured 2.4x slower than the folded FMA path, so reduced operand
precision buys nothing here, and the results stay at least as accurate as the reference's modes
(tests/test_precision_gpu.py checks both switches against the reference's tolerances).

``check_device_errors`` (no counterpart in the reference) makes every DWT call synchronise and
read the device error word afterwards, raising ``RuntimeError`` if a streaming kernel gave up
waiting on an asynchronous copy (its outputs are then incomplete).  Off by default: the check
costs a device synchronisation per call.  Without it, callers that need the guarantee poll
``fdwt_device_error()`` (``_lib.device_error()``) themselves.
"""

allow_tf32: bool = False
allow_bf16: bool = False
check_device_errors: bool = False
