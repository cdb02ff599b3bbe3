"""CPU oracle for the LayerBatch hot path.  TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference's own algorithm for the two hot-path
operators (the Qwen3.5 sparse-MoE block and the paged attention + gated o_proj tail).
It is the checker, never the thing measured or shipped: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs may import it.  The
product path (``layerbatch_b200``) never imports it and fails loudly when its CUDA
library is missing.

Parity is pinned: ``tests/test_oracle_golden.py`` checks these functions against golden
vectors produced by running the reference's own torch modules on seeded inputs
(``tests/golden/make_golden.py``).
"""
