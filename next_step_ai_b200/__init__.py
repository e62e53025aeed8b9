"""B200-native blockwise-sparse NF4 decode MLP (drop-in for next_step_ai's
``exact_blockwise_sparse`` path).

Public API:
  route_sparse_mlp, sparse_mlp_decode, decode_gathered, decode_gathered_rows, union_decode
  RouterWeights, SparseMlpWeights
  triton_sparse_mlp (drop-in module with the reference's function names)
"""
from .mlp import (decode_gathered, decode_gathered_rows, route_sparse_mlp, sparse_mlp_decode,  # noqa: F401
                  union_decode)
from .weights import RouterWeights, SparseMlpWeights  # noqa: F401

SPARSE_MLP_EXECUTION = "exact_blockwise_sparse"
SPARSE_MLP_EXECUTION_ALIASES = {"exact_intermediate_sparse": SPARSE_MLP_EXECUTION}
