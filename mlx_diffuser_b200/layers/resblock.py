"""The TRELLIS sparse residual block around the convolutions, fused for sm_100a.

Drop-in for ``_SparseResBlock3D`` (``src/mlx_diffuser/models/trellis_slat.py:43-92``) with its
helpers ``LayerNorm32`` (``src/mlx_diffuser/layers/trellis.py:16-43``) and ``SparseLinear``
(``src/mlx_diffuser/layers/trellis_sparse.py:13-30``): same constructor arguments, attribute
names (``norm1``, ``norm2``, ``conv1``, ``conv2``, ``emb_layers``, ``skip_connection``) and
initialisation (``conv2`` zeroed). The forward pass is the reference's, with its element-wise
steps fused:

    reference                                   here
    h = silu(norm1(x))                          one sv_rownorm pass
    h = conv1(h)                                tcgen05 conv
    h = silu(norm2(h) * (1 + scale) + shift)    one sv_rownorm pass (batch-indexed modulation)
    out = conv2(h) + skip(x)                    tcgen05 conv, skip added in its epilogue

Every fused step computes in fp32 and rounds once, where the reference rounds to the feature
type after each step; results agree within the half-precision tolerance.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..kernels.norm import row_norm
from .sparse import SparseConv3D, SparseTensor, sparse_downsample, sparse_upsample


class LayerNorm32(nn.Module):
    """LayerNorm computed in fp32 and cast back to the input dtype, eps 1e-6; the affine
    weight and bias are fp32 (``src/mlx_diffuser/layers/trellis.py:16-43``)."""

    def __init__(self, dim: int, *, affine: bool, eps: float = 1e-6):
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.affine = affine
        if affine:
            self.register_buffer("weight", torch.ones(dim, dtype=torch.float32))
            self.register_buffer("bias", torch.zeros(dim, dtype=torch.float32))
        else:
            self.weight = None
            self.bias = None

    def forward(self, x: torch.Tensor, *, silu: bool = False) -> torch.Tensor:
        return row_norm(x, weight=self.weight, bias=self.bias, eps=self.eps, silu=silu)


class SparseLinear(nn.Module):
    """Linear projection of the feature rows (``src/mlx_diffuser/layers/trellis_sparse.py:
    13-30``): ``x.features @ weight.T + bias``, uniform init in ±1/sqrt(in)."""

    def __init__(self, input_dims: int, output_dims: int, bias: bool = True):
        super().__init__()
        bound = math.sqrt(1.0 / input_dims)
        self.register_buffer("weight", torch.empty(output_dims, input_dims).uniform_(-bound, bound))
        if bias:
            self.register_buffer("bias", torch.zeros(output_dims))
        else:
            self.bias = None

    def project(self, features: torch.Tensor) -> torch.Tensor:
        w = self.weight.to(device=features.device, dtype=features.dtype)
        b = None if self.bias is None else self.bias.to(device=features.device,
                                                        dtype=features.dtype)
        return F.linear(features, w, b)

    def forward(self, x: SparseTensor) -> SparseTensor:
        return x.replace(self.project(x.features))


class SparseResBlock3D(nn.Module):
    """``_SparseResBlock3D`` (``src/mlx_diffuser/models/trellis_slat.py:43-92``), fused."""

    def __init__(
        self,
        channels: int,
        emb_channels: int,
        *,
        out_channels: int | None = None,
        downsample: bool = False,
        upsample: bool = False,
        use_metal: bool = True,
    ):
        super().__init__()
        if downsample and upsample:
            raise ValueError("a sparse residual block cannot downsample and upsample")
        self.out_channels = out_channels or channels
        self.downsample = downsample
        self.upsample = upsample
        self.norm1 = LayerNorm32(channels, affine=True)
        self.norm2 = LayerNorm32(self.out_channels, affine=False)
        self.conv1 = SparseConv3D(channels, self.out_channels, 3, use_metal=use_metal)
        self.conv2 = SparseConv3D(self.out_channels, self.out_channels, 3, use_metal=use_metal)
        self.conv2.conv.weight = torch.zeros_like(self.conv2.conv.weight)
        self.conv2.conv.bias = torch.zeros_like(self.conv2.conv.bias)
        self.emb_layers = nn.ModuleList([nn.SiLU(), nn.Linear(emb_channels, 2 * self.out_channels)])
        self.skip_connection = (
            SparseLinear(channels, self.out_channels) if channels != self.out_channels else None
        )

    def forward(self, x: SparseTensor, emb: torch.Tensor) -> SparseTensor:
        layer = self.emb_layers[1]
        proj = F.linear(F.silu(emb.to(layer.weight.dtype)), layer.weight, layer.bias)
        scale, shift = torch.chunk(proj.to(x.dtype), 2, dim=-1)
        if self.downsample:
            x = sparse_downsample(x, 2)
        elif self.upsample:
            x = sparse_upsample(x, 2)
        a = self.norm1(x.features, silu=True)
        h = self.conv1(x.replace(a))
        b = row_norm(h.features, scale=scale, shift=shift, coords=x.coords,
                     batch_size=x.batch_size, silu=True, eps=self.norm2.eps)
        skip = self.skip_connection.project(x.features) if self.skip_connection is not None \
            else x.features
        return self.conv2(h.replace(b), residual=skip)

    def cast_torso(self, dtype: torch.dtype) -> None:
        self.conv1.cast_dtype(dtype)
        self.conv2.cast_dtype(dtype)
        self.emb_layers[1].to(dtype)
        if self.skip_connection is not None:
            self.skip_connection.weight = self.skip_connection.weight.to(dtype)
            if self.skip_connection.bias is not None:
                self.skip_connection.bias = self.skip_connection.bias.to(dtype)


__all__ = ["LayerNorm32", "SparseLinear", "SparseResBlock3D"]
