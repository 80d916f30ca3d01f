"""Sparse voxel tensors and the TRELLIS sparse conv / pooling primitives, on sm_100a.

Drop-in for the sparse-voxel path of ``mlx_diffuser.layers.sparse``
(``src/mlx_diffuser/layers/sparse.py:23-295``): ``SparseTensor``, ``build_neighbor_map``,
``SparseConv3D``, ``sparse_downsample`` and ``sparse_upsample`` keep the reference's names,
arguments, cache keys and errors. Features and coordinates are CUDA ``torch.Tensor``s (any
DLPack array is borrowed); every topology and feature computation runs in ``libsparsevox.so``.

Differences that are deliberate:
* ``build_neighbor_map`` and ``sparse_downsample`` run on the GPU instead of host NumPy; their
  integer outputs are bit-identical to the reference's.
* ``SparseConv3D`` hands the spconv ``(O, k, k, k, I)`` weight to the kernel as is (the
  reference transposes it to ``(k^3, I, O)`` on every call, ``:224-226``) and caches, next to
  the neighbour map, a row schedule that groups rows with equal neighbour masks.
* There is no training-mode fallback (``:233``): the module is inference-only.
"""

from __future__ import annotations

import ctypes
import dataclasses
import math
from typing import Any

import numpy as np
import torch
from torch import nn

from .. import _native as N
from ..kernels.sparse import conv3d_forward


def _triple(value, what: str) -> tuple[int, int, int]:
    if isinstance(value, int):
        return (value, value, value)
    out = tuple(int(v) for v in value)
    if len(out) != 3:
        raise ValueError(f"sparse submanifold kernels must have three odd dimensions ({what})")
    return out  # type: ignore[return-value]


@dataclasses.dataclass
class SparseTensor:
    """Minimal sparse tensor shared by TRELLIS flow and representation decoders.

    ``coords`` are int32 rows ``(batch, x, y, z)``; ``features`` hold one row per coordinate.
    ``cache`` is shared by every tensor derived through :meth:`replace` and holds the
    neighbour maps (``neighbors_{k}_{dilation}_{scale}``) and down/upsample inverses
    (``upsample_{factor}_{scale}``), as in ``src/mlx_diffuser/layers/sparse.py:23-143``.
    """

    features: torch.Tensor
    coords: torch.Tensor
    batch_size: int | None = None
    spatial_shape: tuple[int, int, int] | None = None
    scale: tuple[int, int, int] = (1, 1, 1)
    cache: dict[str, Any] = dataclasses.field(default_factory=dict, repr=False)

    def __post_init__(self) -> None:
        self.features = N.as_tensor(self.features)
        self.coords = N.as_tensor(self.coords)
        if self.features.ndim < 2:
            raise ValueError("features must have shape (N, channels...)")
        if self.coords.ndim != 2 or self.coords.shape[1] != 4:
            raise ValueError(f"coords must have shape (N, 4), got {tuple(self.coords.shape)}")
        if self.features.shape[0] != self.coords.shape[0]:
            raise ValueError("features and coords must contain the same number of points")
        if self.coords.dtype != torch.int32:
            self.coords = self.coords.to(torch.int32)
        if self.batch_size is None:
            self.batch_size = (
                int(self.coords[:, 0].max().item()) + 1 if self.coords.shape[0] else 0
            )
        if self.spatial_shape is None:
            if self.coords.shape[0]:
                maximum = self.coords[:, 1:].max(dim=0).values.to(torch.int64).cpu().tolist()
                self.spatial_shape = (maximum[0] + 1, maximum[1] + 1, maximum[2] + 1)
            else:
                self.spatial_shape = (0, 0, 0)

    @property
    def feats(self) -> torch.Tensor:
        """Alias used by the original TRELLIS sparse modules."""

        return self.features

    @property
    def shape(self) -> tuple[int, ...]:
        assert self.batch_size is not None
        return (self.batch_size, *self.features.shape[1:])

    @property
    def dtype(self) -> torch.dtype:
        return self.features.dtype

    @property
    def num_points(self) -> int:
        return self.features.shape[0]

    def replace(
        self,
        features: torch.Tensor,
        coords: torch.Tensor | None = None,
        *,
        batch_size: int | None = None,
        spatial_shape: tuple[int, int, int] | None = None,
        scale: tuple[int, int, int] | None = None,
    ) -> SparseTensor:
        return SparseTensor(
            features,
            self.coords if coords is None else coords,
            self.batch_size if batch_size is None else batch_size,
            self.spatial_shape if spatial_shape is None else spatial_shape,
            self.scale if scale is None else scale,
            self.cache,
        )

    def batch_layout(self) -> tuple[slice, ...]:
        batch = self.coords[:, 0].to(torch.int64).cpu().numpy()
        assert self.batch_size is not None
        counts = np.bincount(batch, minlength=self.batch_size)
        offsets = np.concatenate([[0], np.cumsum(counts)])
        return tuple(slice(int(offsets[i]), int(offsets[i + 1])) for i in range(self.batch_size))

    def _broadcast_other(self, other: Any) -> Any:
        if isinstance(other, SparseTensor):
            if other.coords.shape != self.coords.shape:
                raise ValueError("sparse tensors must have matching coordinates")
            return other.features
        if (
            isinstance(other, torch.Tensor)
            and other.ndim >= 1
            and other.shape[0] == self.batch_size
        ):
            return other[self.coords[:, 0].long()]
        return other

    def __add__(self, other: Any) -> SparseTensor:
        return self.replace(self.features + self._broadcast_other(other))

    def __radd__(self, other: Any) -> SparseTensor:
        return self + other

    def __sub__(self, other: Any) -> SparseTensor:
        return self.replace(self.features - self._broadcast_other(other))

    def __rsub__(self, other: Any) -> SparseTensor:
        return self.replace(self._broadcast_other(other) - self.features)

    def __mul__(self, other: Any) -> SparseTensor:
        return self.replace(self.features * self._broadcast_other(other))

    def __rmul__(self, other: Any) -> SparseTensor:
        return self * other

    def __truediv__(self, other: Any) -> SparseTensor:
        return self.replace(self.features / self._broadcast_other(other))

    def astype(self, dtype: torch.dtype) -> SparseTensor:
        return self.replace(self.features.to(dtype))

    def dense(self, fill_value: float = 0.0) -> torch.Tensor:
        assert self.batch_size is not None and self.spatial_shape is not None
        out = torch.full(
            (self.batch_size, *self.spatial_shape, *self.features.shape[1:]),
            fill_value,
            dtype=self.features.dtype,
            device=self.features.device,
        )
        index = tuple(self.coords[:, i].long() for i in range(4))
        return out.index_put_(index, self.features, accumulate=True)


def build_neighbor_map(
    coords,
    kernel_size: int | tuple[int, int, int],
    dilation: int | tuple[int, int, int] = 1,
    *,
    table_slots: int | None = None,
) -> torch.Tensor:
    """Build the input-point map for submanifold cross-correlation.

    Same result as ``src/mlx_diffuser/layers/sparse.py:146-175``: ``(N, kD*kH*kW)`` int32 where
    column ``k`` enumerates offsets with the first spatial column outermost, a missing
    neighbour is ``-1`` and duplicate coordinate rows resolve to the last such row. Runs on
    the coordinates' CUDA device. ``table_slots`` overrides the hash-table size (a power of
    two); an undersized table raises instead of returning a partial map.
    """

    kernel = _triple(kernel_size, "kernel_size")
    dilations = _triple(dilation, "dilation")
    if any(k % 2 == 0 for k in kernel):
        raise ValueError("sparse submanifold kernels must have three odd dimensions")
    coords = N.as_tensor(coords)
    if coords.ndim != 2 or coords.shape[1] != 4:
        raise ValueError(f"coords must have shape (N, 4), got {tuple(coords.shape)}")
    N.require_cuda(coords, "coords")
    coords = coords.to(torch.int32).contiguous()
    n = coords.shape[0]
    kvol = kernel[0] * kernel[1] * kernel[2]
    out = torch.empty((n, kvol), dtype=torch.int32, device=coords.device)
    if n == 0:
        return out
    lib = N.load()
    slots = int(table_slots) if table_slots is not None else int(lib.sv_kmap_table_slots(n))
    ws_bytes = lib.sv_kmap_workspace_bytes(slots)
    ws = N.workspace(ws_bytes, coords.device)
    int3 = ctypes.c_int * 3
    status = N.status_word(coords.device)
    rc = lib.sv_kmap_build(
        coords.data_ptr(), n, int3(*kernel), int3(*dilations), out.data_ptr(), slots,
        ws.data_ptr(), ws_bytes, status.data_ptr(), N.stream(coords.device),
    )
    N.check(rc, "build_neighbor_map")
    if table_slots is not None:
        N.check_device_status(coords.device)
    return out


def conv_row_order(neighbors: torch.Tensor) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """Schedule for the tensor-core convolution: ``(row_order, tile_order)``. Rows are grouped
    by neighbour mask; the 128-row tiles are listed most expensive first. ``(None, None)`` when
    the kernel volume exceeds 32 (the convolution then runs in plain row order)."""

    n, kvol = neighbors.shape
    if n == 0 or kvol > 32:
        return None, None
    lib = N.load()
    dev = neighbors.device
    order = torch.empty(n, dtype=torch.int32, device=dev)
    tiles = torch.empty(int(lib.sv_conv_plan_tiles(n)), dtype=torch.int32, device=dev)
    ws_bytes = lib.sv_conv_plan_workspace_bytes(n)
    ws = N.workspace(ws_bytes, dev)
    rc = lib.sv_conv_plan(neighbors.data_ptr(), n, kvol, order.data_ptr(), tiles.data_ptr(),
                          ws.data_ptr(), ws_bytes, N.stream(dev))
    N.check(rc, "conv row schedule")
    return order, tiles


class _SparseConv3DCore(nn.Module):
    """Parameter holder matching spconv's ``(O, kD, kH, kW, I)`` layout
    (``src/mlx_diffuser/layers/sparse.py:178-193``): uniform init in ±1/sqrt(I*k^3), zero bias.
    Parameters are buffers so that plain tensors can be assigned, as mlx_diffuser does."""

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, bias: bool):
        super().__init__()
        kernel_volume = kernel_size**3
        bound = 1.0 / math.sqrt(in_channels * kernel_volume)
        self.register_buffer(
            "weight",
            torch.empty(out_channels, kernel_size, kernel_size, kernel_size, in_channels).uniform_(
                -bound, bound
            ),
        )
        if bias:
            self.register_buffer("bias", torch.zeros(out_channels))
        else:
            self.register_buffer("_bias", torch.zeros(out_channels))


class SparseConv3D(nn.Module):
    """Submanifold Conv3D (``src/mlx_diffuser/layers/sparse.py:196-242``) on sm_100a."""

    def __init__(
        self,
        in_channels: int,
        out_channels: int,
        kernel_size: int = 3,
        *,
        dilation: int = 1,
        bias: bool = True,
        use_metal: bool = True,
    ):
        super().__init__()
        if kernel_size % 2 == 0:
            raise ValueError("SparseConv3D requires an odd kernel_size")
        self.kernel_size = kernel_size
        self.dilation = dilation
        self.use_metal = use_metal  # accepted for compatibility; the CUDA kernels always run
        self.algo = N.SV_CONV_AUTO
        self.conv = _SparseConv3DCore(in_channels, out_channels, kernel_size, bias)
        self._operand_cache: tuple[Any, torch.Tensor, torch.Tensor] | None = None

    def _operands(self, device: torch.device, dtype: torch.dtype):
        weight = self.conv.weight
        bias = self.conv.bias if hasattr(self.conv, "bias") else self.conv._bias
        if (
            weight.device == device
            and weight.dtype == dtype
            and weight.is_contiguous()
            and bias.device == device
            and bias.dtype == dtype
        ):
            return weight, bias
        key = (weight.data_ptr(), weight._version, bias.data_ptr(), bias._version, device, dtype)
        if self._operand_cache is None or self._operand_cache[0] != key:
            self._operand_cache = (
                key,
                weight.to(device=device, dtype=dtype).contiguous(),
                bias.to(device=device, dtype=dtype).contiguous(),
            )
        return self._operand_cache[1], self._operand_cache[2]

    def forward(self, x: SparseTensor) -> SparseTensor:
        key = f"neighbors_{self.kernel_size}_{self.dilation}_{x.scale}"
        neighbors = x.cache.get(key)
        if neighbors is None:
            neighbors = build_neighbor_map(x.coords, self.kernel_size, self.dilation)
            x.cache[key] = neighbors
        plan_key = f"conv_rows_{self.kernel_size}_{self.dilation}_{x.scale}"
        if plan_key not in x.cache:
            x.cache[plan_key] = conv_row_order(neighbors)
        features = x.features
        if features.ndim != 2:
            raise ValueError(f"features must be 2D, got {tuple(features.shape)}")
        N.require_cuda(features, "features")
        weight, bias = self._operands(features.device, features.dtype)
        o, _, _, _, i = weight.shape
        if features.shape[1] != i or neighbors.shape[0] != features.shape[0]:
            raise ValueError(
                "weights must have shape "
                f"({neighbors.shape[1]}, {features.shape[1]}, Cout), got "
                f"({self.kernel_size**3}, {i}, {o})"
            )
        row_order, tile_order = x.cache[plan_key]
        out = conv3d_forward(
            features.contiguous(), neighbors, weight, N.SV_WEIGHT_OKI, bias, o,
            row_order=row_order, tile_order=tile_order, algo=self.algo,
        )
        return x.replace(out)

    def cast_dtype(self, dtype: torch.dtype) -> None:
        self.conv.weight = self.conv.weight.to(dtype)
        if hasattr(self.conv, "bias"):
            self.conv.bias = self.conv.bias.to(dtype)
        else:
            self.conv._bias = self.conv._bias.to(dtype)


def sparse_downsample(x: SparseTensor, factor: int = 2) -> SparseTensor:
    """Average-pool occupied coordinates and cache the inverse for upsampling
    (``src/mlx_diffuser/layers/sparse.py:245-284``): coords become ``unique(coords // f)`` in
    lexicographic order, features ``sum / (count + 1)``."""

    if factor < 1:
        raise ValueError("factor must be positive")
    coords = x.coords.contiguous()
    N.require_cuda(coords, "coords")
    dev = coords.device
    n = coords.shape[0]
    lib = N.load()
    new_coords = torch.empty((n, 4), dtype=torch.int32, device=dev)
    inverse = torch.empty(n, dtype=torch.int32, device=dev)
    sorted_rows = torch.empty(n, dtype=torch.int32, device=dev)
    seg = torch.empty(n + 1, dtype=torch.int32, device=dev)
    m_out = ctypes.c_int64(0)
    ws_bytes = lib.sv_downsample_workspace_bytes(n)
    ws = N.workspace(ws_bytes, dev)
    rc = lib.sv_downsample_coords(
        coords.data_ptr(), n, factor, new_coords.data_ptr(), inverse.data_ptr(),
        sorted_rows.data_ptr(), seg.data_ptr(), ctypes.byref(m_out), ws.data_ptr(), ws_bytes,
        N.stream(dev),
    )
    N.check(rc, "sparse_downsample")
    m = int(m_out.value)
    feats = x.features
    trailing = feats.shape[1:]
    flat = feats.reshape(n, math.prod(trailing)).contiguous()
    if flat.dtype not in N.DTYPE_CODE:
        flat = flat.to(torch.float32)
    pooled = torch.empty((m, flat.shape[1]), dtype=flat.dtype, device=dev)
    rc = lib.sv_downsample_features(
        flat.data_ptr(), n, flat.shape[1], N.DTYPE_CODE[flat.dtype], sorted_rows.data_ptr(),
        seg.data_ptr(), m, pooled.data_ptr(), N.stream(dev),
    )
    N.check(rc, "sparse_downsample")
    features = pooled.reshape(m, *trailing).to(feats.dtype)
    scale = tuple(value * factor for value in x.scale)
    scale = (scale[0], scale[1], scale[2])
    source_shape = x.spatial_shape or (0, 0, 0)
    spatial_shape = (
        math.ceil(source_shape[0] / factor),
        math.ceil(source_shape[1] / factor),
        math.ceil(source_shape[2] / factor),
    )
    out = SparseTensor(features, new_coords[:m], x.batch_size, spatial_shape, scale, x.cache)
    out.cache[f"upsample_{factor}_{scale}"] = (x.coords, inverse, x.spatial_shape, x.scale)
    return out


def sparse_upsample(x: SparseTensor, factor: int = 2) -> SparseTensor:
    """Nearest-neighbor inverse of :func:`sparse_downsample`
    (``src/mlx_diffuser/layers/sparse.py:287-295``)."""

    key = f"upsample_{factor}_{x.scale}"
    cached = x.cache.get(key)
    if cached is None:
        raise ValueError("sparse_upsample must be paired with a cached sparse_downsample")
    coords, inverse, spatial_shape, scale = cached
    feats = x.features
    N.require_cuda(feats, "features")
    m = feats.shape[0]
    n = inverse.shape[0]
    flat = feats.reshape(m, math.prod(feats.shape[1:])).contiguous()
    out = torch.empty((n, flat.shape[1]), dtype=flat.dtype, device=flat.device)
    # the gather copies rows of bytes: describe any row as float32 / 16-bit words
    row_bytes = flat.shape[1] * flat.element_size()
    if flat.dtype in N.DTYPE_CODE:
        words, code = flat.shape[1], N.DTYPE_CODE[flat.dtype]
    elif row_bytes % 4 == 0:
        words, code = row_bytes // 4, N.DTYPE_CODE[torch.float32]
    elif row_bytes % 2 == 0:
        words, code = row_bytes // 2, N.DTYPE_CODE[torch.float16]
    else:
        raise ValueError(f"sparse_upsample: unsupported feature dtype {flat.dtype}")
    lib = N.load()
    rc = lib.sv_upsample_features(
        flat.data_ptr(), m, words, code, inverse.data_ptr(), n, out.data_ptr(),
        N.status_word(flat.device).data_ptr(), N.stream(flat.device),
    )
    N.check(rc, "sparse_upsample")
    features = out.reshape(n, *feats.shape[1:])
    return SparseTensor(features, coords, x.batch_size, spatial_shape, scale, x.cache)


__all__ = [
    "SparseConv3D",
    "SparseTensor",
    "build_neighbor_map",
    "sparse_downsample",
    "sparse_upsample",
]
