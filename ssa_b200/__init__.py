"""ssa_b200 -- the sparse-attention hot path of daedalus/SSA on B200 (sm_100a).

Drop-in API: the names below match the reference module `sparse_attention`.
The graph build and gather attention run as hand-written CUDA kernels in
libssa_b200.so (C ABI: include/ssa_b200.h); PyTorch supplies device memory,
streams, the q/k/v/o projections and torch.distributed.
"""
from .attention import (  # noqa: F401
    SSAConfig,
    SubquadraticRegimeTracker,
    WindowGraphBuilder,
    GlobalGraphBuilder,
    LSHGraphBuilder,
    merge_neighbors,
    sparse_gather_attention,
    SparseAttention,
    SparseTransformerLayer,
    SparseTransformer,
    neighbor_overlap,
    measure_cross_layer_overlap,
    CachedGraphSparseTransformer,
)

__all__ = [
    "SSAConfig", "SubquadraticRegimeTracker", "WindowGraphBuilder", "GlobalGraphBuilder",
    "LSHGraphBuilder", "merge_neighbors", "sparse_gather_attention", "SparseAttention",
    "SparseTransformerLayer", "SparseTransformer", "neighbor_overlap",
    "measure_cross_layer_overlap", "CachedGraphSparseTransformer",
]
