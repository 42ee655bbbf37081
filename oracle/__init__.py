"""TEST INFRASTRUCTURE ONLY -- the CPU oracle the CUDA path is checked against.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import this package, and
only as the checker / the timed CPU baseline.  The product path (``mace_mps_kernels_b200``) never imports it and has
no CPU fallback.

Contents (float64 numpy restatements of the reference's algorithm for the hot path, each function citing the
reference file:line it follows; reference = Yike-Ye/mace-mps-kernels v0.1.0):
  conv_ref   probe of the path coefficients, csr_by, conv forward / backward semantics
  sc_ref     polynomial coefficients of the symmetric contraction, term list, forward / backward semantics

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own Python (ConvSpec, SCSpec, _poly_coeffs,
csr_by) and the reference's generated kernels (compiled as C++ on the CPU) on stand-in models and small random
inputs; ``tests/test_oracle_golden.py`` checks this oracle against those committed fixtures.
"""
