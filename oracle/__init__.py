"""CPU oracle for the blockwise-sparse NF4 decode MLP.

TEST INFRASTRUCTURE ONLY.  This package restates, in numpy, the reference
(andott28/next_step_ai) algorithm for the exact blockwise-sparse decode MLP:
the learned-basis router, the active-block layout, the NF4 dequant + matmul
fallback, the Triton kernels' own index arithmetic, and the VRAM hot-block
bank policy.  Every function cites the reference file:line it follows.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import it, and only as the checker (or, for the baseline, as the timed
CPU port of the reference path).  The product package never imports it.

Parity pin: the oracle is checked against golden vectors produced by the
reference's own code run in the build container (``tests/golden/make_golden.py``):
``StreamingLlamaRuntime._route_sparse_mlp`` / ``_build_sparse_active_layout`` /
``_plan_fixed_capacity_bank_update`` / ``_record_hot_cache_calibration_blocks`` /
``_load_down_proj_cold_cols`` executed on CPU, and the reference's Triton
kernels executed by Triton's CPU interpreter.
"""
