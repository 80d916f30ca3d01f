"""B200-native (sm_100a) TRELLIS sparse-voxel path: the drop-in for mlx_diffuser's
``SparseTensor`` / ``build_neighbor_map`` / ``SparseConv3D`` / ``sparse_conv3d`` /
``sparse_downsample`` / ``sparse_upsample``, backed by ``libsparsevox.so``."""

from ._native import check_device_status
from .kernels.sparse import sparse_conv3d
from .layers.sparse import (
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
    "check_device_status",
    "sparse_conv3d",
    "sparse_downsample",
    "sparse_upsample",
]
