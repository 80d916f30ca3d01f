"""Sparse submanifold convolution over a precomputed neighbour map, on sm_100a.

Drop-in for ``mlx_diffuser.kernels.sparse`` (``src/mlx_diffuser/kernels/sparse.py``): the same
function name, arguments, validation and errors, computing what the reference's Metal kernel
computes (``:9-36``) -- fp32 accumulation, one rounding to the feature dtype -- with the
library's tcgen05 kernel (fp16/bf16 with Cin % 32 == 0 and Cout % 32 == 0) or its CUDA-core
kernel (everything else). ``use_metal`` is accepted for signature compatibility; there is one
(CUDA) implementation and no CPU fallback.
"""

from __future__ import annotations

import torch

from .. import _native as N


def _check_shapes(features, neighbors, weights, bias) -> None:
    # validation of src/mlx_diffuser/kernels/sparse.py:78-88, same messages
    if features.ndim != 2:
        raise ValueError(f"features must be 2D, got {tuple(features.shape)}")
    if neighbors.ndim != 2 or neighbors.shape[0] != features.shape[0]:
        raise ValueError("neighbors must have shape (N, kernel_volume)")
    if weights.ndim != 3 or tuple(weights.shape[:2]) != (neighbors.shape[1], features.shape[1]):
        raise ValueError(
            "weights must have shape "
            f"({neighbors.shape[1]}, {features.shape[1]}, Cout), got {tuple(weights.shape)}"
        )
    if tuple(bias.shape) != (weights.shape[2],):
        raise ValueError(f"bias must have shape ({weights.shape[2]},), got {tuple(bias.shape)}")


def conv3d_forward(
    features: torch.Tensor,
    neighbors: torch.Tensor,
    weight: torch.Tensor,
    layout: int,
    bias: torch.Tensor | None,
    cout: int,
    *,
    row_order: torch.Tensor | None = None,
    tile_order: torch.Tensor | None = None,
    algo: int = N.SV_CONV_AUTO,
    out: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
) -> torch.Tensor:
    """Call ``sv_conv3d_forward_residual``. Tensors must already be contiguous, on one CUDA
    device, and share the feature dtype (``neighbors`` int32); ``layout`` is SV_WEIGHT_KIO or
    _OKI. ``row_order`` / ``tile_order`` are the schedule from :func:`conv_row_order`.
    ``residual`` ([n, cout], optional, may be ``out``) is added to the result before rounding."""

    n, cin = features.shape
    kvol = neighbors.shape[1]
    dev = features.device
    if out is None:
        out = torch.empty((n, cout), dtype=features.dtype, device=dev)
    if n == 0 or cout == 0:
        return out
    dcode = N.DTYPE_CODE[features.dtype]
    lib = N.load()
    ws_bytes = lib.sv_conv3d_workspace_bytes(n, cin, cout, kvol, dcode, layout, algo)
    ws = N.workspace(ws_bytes, dev) if ws_bytes else None
    if residual is not None and (tuple(residual.shape) != (n, cout)
                                 or residual.dtype != features.dtype
                                 or not residual.is_contiguous()):
        raise ValueError(f"residual must be a contiguous ({n}, {cout}) {features.dtype} tensor")
    rc = lib.sv_conv3d_forward_residual(
        features.data_ptr(),
        n,
        cin,
        neighbors.data_ptr(),
        kvol,
        N.ptr(row_order),
        N.ptr(tile_order),
        weight.data_ptr(),
        layout,
        N.ptr(bias),
        N.ptr(residual),
        cout,
        dcode,
        out.data_ptr(),
        algo,
        N.ptr(ws),
        ws_bytes,
        N.status_word(dev).data_ptr(),
        N.stream(dev),
    )
    N.check(rc, "sparse_conv3d")
    return out


def sparse_conv3d(
    features,
    neighbors,
    weights,
    bias,
    *,
    use_metal: bool = True,
) -> torch.Tensor:
    """Apply a submanifold sparse Conv3D over a precomputed neighbor map.

    Args:
        features: Point features ``(N, Cin)`` (float32, float16 or bfloat16, on CUDA).
        neighbors: Input row for every ``(point, kernel_offset)``, shape ``(N, K)``;
            ``-1`` denotes an empty neighbor.
        weights: Kernel weights ``(K, Cin, Cout)``.
        bias: Output bias ``(Cout,)``.
        use_metal: accepted for compatibility with mlx_diffuser; ignored.

    Returns ``(N, Cout)`` in the feature dtype.
    """

    del use_metal
    features = N.as_tensor(features)
    neighbors = N.as_tensor(neighbors)
    weights = N.as_tensor(weights)
    bias = N.as_tensor(bias)
    _check_shapes(features, neighbors, weights, bias)
    N.require_cuda(features, "features")
    if features.dtype not in N.DTYPE_CODE:
        raise ValueError(f"unsupported feature dtype {features.dtype}")
    dev, dtype = features.device, features.dtype
    if neighbors.dtype != torch.int32:
        neighbors = neighbors.to(torch.int32)
    n, cout = features.shape[0], weights.shape[2]
    if n * cout == 0:
        return torch.zeros((n, cout), dtype=dtype, device=dev)
    features = features.contiguous()
    neighbors = neighbors.to(dev).contiguous()
    weights = weights.to(device=dev, dtype=dtype).contiguous()
    bias = bias.to(device=dev, dtype=dtype).contiguous()
    return conv3d_forward(features, neighbors, weights, N.SV_WEIGHT_KIO, bias, cout)


__all__ = ["sparse_conv3d"]
