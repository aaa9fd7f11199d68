"""CPU oracle for the batch-one decode path (TEST INFRASTRUCTURE ONLY).

This package restates, in plain PyTorch on the CPU, the arithmetic of the
reference engine's decode path (maokner/moe-inference-engine,
``src/moe_engine/model.py``).  It is the checker for the CUDA kernels: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  The product package
``moe_engine`` never imports it and has no CPU fallback into it.

Parity pin: ``tests/golden/make_golden.py`` runs the unmodified reference
(reference architecture: LayerNorm, learned positions, biased GELU experts)
and stores its outputs under ``tests/golden/``; ``tests/test_oracle_golden.py``
checks this restatement against them.  The BASELINE architecture differs by
three documented substitutions (RMSNorm, RoPE, SwiGLU), each pinned against an
independent formulation in the same test file.
"""

from .minimoe import *  # noqa: F401,F403
