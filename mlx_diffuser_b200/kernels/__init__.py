"""CUDA sparse kernels (drop-in for ``mlx_diffuser.kernels``)."""

from .sparse import sparse_conv3d

__all__ = ["sparse_conv3d"]
