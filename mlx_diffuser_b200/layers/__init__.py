"""Sparse-voxel layers (drop-in for ``mlx_diffuser.layers.sparse``)."""

from .sparse import (
    SparseConv3D,
    SparseTensor,
    build_neighbor_map,
    sparse_downsample,
    sparse_upsample,
)

__all__ = [
    "SparseConv3D",
    "SparseTensor",
    "build_neighbor_map",
    "sparse_downsample",
    "sparse_upsample",
]
