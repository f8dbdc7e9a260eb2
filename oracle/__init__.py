"""CPU oracle for the adallm_b200 hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain numpy / eager CPU torch, the arithmetic of the
reference runtime (Kukuskas/AdaLLMv2, package ``adallm``) for the two decode
hot paths: the NVFP4 linear op and FP8 paged decode attention, plus the FP8
KV-cache store, RMSNorm and rotary embedding.  Every function cites the
reference file:line it follows.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or as the timed CPU baseline.  The product path (``adallm_b200``)
never imports it and fails loudly when its CUDA library is missing.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own Python
functions (imported from a checkout of the reference) on seeded inputs and
stores the results under ``tests/golden/*.npz``; ``tests/test_oracle_golden.py``
checks every oracle function against those fixtures.
"""
