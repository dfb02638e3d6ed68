"""CPU oracle for the LightningRouter MoE-layer hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory: it is read by ``tests/``, by ``__graft_entry__.smoke()`` (as the
checker) and by ``bench.py``'s CPU-baseline / reference arm.  The product path
(``lightning_router``) fails loudly when its CUDA extension is missing and
never falls back to this code.

Parity is pinned against the reference itself: ``tests/golden/make_golden.py``
imports the reference package (read-only) in the build container, runs its
own PyTorch code (and its Triton kernels under ``TRITON_INTERPRET=1``) on
seeded inputs and commits the results as ``tests/golden/*.npz``;
``tests/test_oracle_golden.py`` checks this oracle against them.
"""

from .moe_oracle import *  # noqa: F401,F403
