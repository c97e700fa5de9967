"""B200-native FlashLog soft-grounding propagation (drop-in for flashlog_kernel).

The names exported here are those of the reference package
(flashlog_kernel/__init__.py); the implementation runs in hand-written sm_100a
kernels behind the C ABI of include/flashlog_b200.h.
"""
from . import dropout, filters, readout  # noqa: F401  (value dropout; filter keys; channel readouts)
from .flashlog_kernel import (  # noqa: F401
    FlashLogDenseMaxFunction,
    FlashLogDenseSumFunction,
    FlashLogFunction,
    FlashLogFunctionSparse3DAllEdgesSum,
    FlashLogFunctionSparse3DTopKMax,
    FlashLogFunctionSparse3DTopKSum,
    Sparse3DNormalizeFunction,
    _compute_active_nodes,
    _dense_topc_state,
    _group_starts_and_counts,
    build_csr_structure,
    configure_flashlog_cpu_threads,
    dense_csr_max,
    dense_csr_sum_cuda,
    normalize_sparse3d,
    prepare_csr_masks,
    sampled_sparse_propagation,
    sparse2d_filtered_ranks_cuda,
    vectorized_operation_csr,
    vectorized_operation_sparse3d_csr_sum,
    vectorized_operation_sparse3d_csr_sum_norm,
    vectorized_operation_sparse3d_fixed_relation,
)

__all__ = [
    "FlashLogFunction",
    "_compute_active_nodes",
    "build_csr_structure",
    "prepare_csr_masks",
    "vectorized_operation_csr",
    "vectorized_operation_sparse3d_csr_sum",
    "vectorized_operation_sparse3d_csr_sum_norm",
    "vectorized_operation_sparse3d_fixed_relation",
]
