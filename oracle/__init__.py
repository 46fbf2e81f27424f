"""CPU oracle for the wavelet filter-bank hot path.

TEST INFRASTRUCTURE ONLY.  This package restates, on the CPU, the algorithm of the
reference's own CPU path (``fdwt/reference.py`` and the torch branches of ``fdwt/cwt.py``
and ``fdwt/layers.py`` of Mousakaa/pytorch_morlet_fdwt).  Only ``tests/``, the ``smoke()``
check of ``__graft_entry__`` and ``bench.py``'s CPU-baseline / reference arm may import it,
and only as the checker or as the timed CPU baseline.  The product package
``pytorch_morlet_fdwt_b200`` never imports it and has no CPU fallback.

Parity status: pinned.  ``tests/golden/make_golden.py`` runs the reference's own CPU path
(imported from its source tree) on seeded inputs and stores the outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this oracle against every fixture.
PyWavelets itself is absent from the build container, so agreement with ``pywt``'s named
filter tables is not pinned here (the fixtures pass explicit filter banks to both sides).

* :mod:`oracle.dwt_oracle` -- every DWT level as an explicit sparse operator matrix built from
  the boundary-extension index map; inverse DWT and all gradients are exact transposes.
* :mod:`oracle.cwt_oracle` -- the Morlet plan, filter synthesis, the a-trous pyramid with an
  explicit tap loop, the fused mixers' definitions; gradients by torch autograd in fp64.
"""
