"""CPU oracle for the sonata_b200 hot paths -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, what the reference (Vishal-Padia/Sonata)
computes on each hot path, so that the CUDA kernels in ``sonata_b200`` can be
checked against it.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg may import it, and only as the checker or the
timed CPU baseline -- the product never calls into it, and the product raises
if its CUDA library is missing instead of falling back to anything here.

Parity is pinned: ``tests/golden/make_golden.py`` imports the reference's own
Python modules (``kernels/fused_snake_conv.py``, ``scripts/fake_quant.py``,
``kernels/bmm.py``'s einsum oracle) in the build container and freezes their
outputs on seeded inputs as ``tests/golden/*.npz``; ``tests/test_oracle.py``
checks every function here against those fixtures.
"""
from .oracle import *  # noqa: F401,F403
