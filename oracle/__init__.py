"""CPU oracle for the Iris-3B denoiser hot path -- TEST INFRASTRUCTURE ONLY.

A plain-PyTorch fp32 restatement of the reference's per-step forward
(``src/iris3b/models/dit.py:283-375`` and the blocks it calls), its per-op
kernel references (``src/iris_metal/kernels.py:314-331,424-426,460-462,
488-489,501-524``), the seeded random-init recipe and the samplers that call
the forward (``src/iris3b/sampling.py:98-138``, ``src/iris3b/flow/solver.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package, and only as the checker (or, for the CPU
baseline, as the thing timed on the host cores). The product package never
imports it.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own code and
stores its outputs under ``tests/golden/``; ``tests/test_oracle.py`` checks
this restatement against those fixtures.
"""
