"""Global precision switches (same names and defaults as the reference's ``fdwt/config.py:17-18``).

``allow_tf32`` and ``allow_bf16`` are read at call time.  The sm_100a kernels of this package
compute every filter-bank contraction with fp32 FMAs for fp32/fp16/bf16 inputs and fp64 FMAs
for fp64 inputs, so both switches are accepted for drop-in compatibility and currently select
the same full-precision kernels (results are at least as accurate as the reference's modes).
"""

allow_tf32: bool = False
allow_bf16: bool = False
