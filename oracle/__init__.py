"""CPU oracle for the DimmerKV attention-over-compressed-cache path.

TEST INFRASTRUCTURE ONLY. This package restates, in numpy, the reference
algorithm of SrikanthBalaaji/Dimmer-KV for the hot path (bit-plane
dequantisation, per-layer key rebuild, attention with values kept in
coefficient space, question-time importance, top-k and refine). Each function
cites the reference file:line it follows (paths inside the reference project).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it, and there only as the
checker or as the timed CPU baseline. The product path (``dimmerkv``) never
imports it and fails loudly when its CUDA library is missing.

Parity of this oracle is pinned against fixtures produced by running the
reference's own Python code on seeded inputs (``tests/golden/make_golden.py``;
checked by ``tests/test_oracle_golden.py``).
"""

from . import codes, planes, attention  # noqa: F401
