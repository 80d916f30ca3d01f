"""Sparse submanifold convolution over a precomputed neighbour map, on sm_100a.

Drop-in for ``mlx_diffuser.kernels.sparse`` (``src/mlx_diffuser/kernels/sparse.py``): the same
function name, arguments, validation and errors, computing what the reference's Metal kernel
computes (``:9-36``) -- fp32 accumulation, one rounding to the feature dtype -- with the
library's tcgen05 kernels when Cin and Cout are multiples of 32 (fp16/bf16 directly, fp32 as
3xTF32; fp16/bf16 also with 8 or 16 channels) or its CUDA-core kernel (everything else). ``use_metal`` is accepted for signature compatibility; there is one
(CUDA) implementation and no CPU fallback.
"""

from __future__ import annotations

import ctypes

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


# sv_conv3d_workspace_bytes by argument tuple (a pure function of the shapes)
_WS_BYTES: dict[tuple, int] = {}


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
    rows: torch.Tensor | None = None,
) -> torch.Tensor:
    """Call ``sv_conv3d_forward_residual``. Tensors must already be contiguous, on one CUDA
    device, and share the feature dtype (``neighbors`` int32); ``layout`` is SV_WEIGHT_KIO or
    _OKI. ``row_order`` / ``tile_order`` are the schedule from :func:`conv_row_order`.
    ``residual`` ([n, cout], optional, may be ``out``) is added to the result before rounding.
    ``rows`` (int32, optional) restricts the output to those rows, computed in that order with
    ``tile_order`` as its tile schedule; the other rows of ``out`` are left untouched."""

    n, cin = features.shape
    kvol = neighbors.shape[1]
    dev = features.device
    if out is None:
        out = torch.empty((n, cout), dtype=features.dtype, device=dev)
    if n == 0 or cout == 0:
        return out
    dcode = N.DTYPE_CODE[features.dtype]
    lib = N.load()
    size_key = (n, cin, cout, kvol, dcode, layout, algo)
    ws_bytes = _WS_BYTES.get(size_key)
    if ws_bytes is None:
        ws_bytes = lib.sv_conv3d_workspace_bytes(n, cin, cout, kvol, dcode, layout, algo)
        if len(_WS_BYTES) > 1024:
            _WS_BYTES.clear()
        _WS_BYTES[size_key] = ws_bytes
    ws = N.workspace(ws_bytes, dev) if ws_bytes else None
    if residual is not None and (tuple(residual.shape) != (n, cout)
                                 or residual.dtype != features.dtype
                                 or not residual.is_contiguous()):
        raise ValueError(f"residual must be a contiguous ({n}, {cout}) {features.dtype} tensor")
    if rows is not None:
        rows = rows.to(device=dev, dtype=torch.int32).contiguous()
        if rows.numel() == 0:
            return out
    rc = lib.sv_conv3d_forward_rows(
        features.data_ptr(),
        n,
        cin,
        neighbors.data_ptr(),
        kvol,
        N.ptr(rows if rows is not None else row_order),
        rows.numel() if rows is not None else n,
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


class DedupPlan:
    """Tile plan of the deduplicated narrow-channel convolution (``sv_conv_dd_plan``) for one
    kernel map: 128-row tiles in Morton order, each with its distinct source rows and a local
    map into them. Built once per map and input width, cached next to the map."""

    def __init__(self, coords: torch.Tensor, neighbors: torch.Tensor, cin: int):
        n, kvol = neighbors.shape
        dev = neighbors.device
        lib = N.load()
        self.n, self.cin = n, cin
        self.nbytes = int(lib.sv_conv_dd_plan_bytes(n, cin))
        self.buffer = torch.empty(max(self.nbytes, 1), dtype=torch.uint8, device=dev)
        if n == 0:
            return
        coords = coords.to(device=dev, dtype=torch.int32).contiguous()
        ws_bytes = lib.sv_conv_dd_plan_workspace_bytes(n)
        ws = N.workspace(ws_bytes, dev)
        rc = lib.sv_conv_dd_plan(coords.data_ptr(), neighbors.data_ptr(), n, kvol, cin,
                                 self.buffer.data_ptr(), self.nbytes, ws.data_ptr(), ws_bytes,
                                 N.status_word(dev).data_ptr(), N.stream(dev))
        N.check(rc, "sparse_conv3d (tile plan)")


def dedup_supported(n: int, cin: int, cout: int, kvol: int, dtype: torch.dtype) -> bool:
    code = N.DTYPE_CODE.get(dtype)
    return code is not None and bool(N.load().sv_conv_dd_supported(n, cin, cout, kvol, code))


def conv3d_forward_dd(features, neighbors, plan: DedupPlan, weight_oki, bias, cout, *,
                      out=None, residual=None) -> torch.Tensor:
    """``sv_conv3d_forward_dd``: the narrow-channel tensor-core convolution over a
    :class:`DedupPlan` (fp16/bf16, 3x3x3, Cin 64 or 128, Cout % 32 == 0). Tensors contiguous
    on one CUDA device, weight in the spconv (Cout, 3, 3, 3, Cin) layout."""

    n, cin = features.shape
    dev = features.device
    if out is None:
        out = torch.empty((n, cout), dtype=features.dtype, device=dev)
    if n == 0 or cout == 0:
        return out
    if plan.n != n or plan.cin != cin:
        raise ValueError("tile plan was built for another map or input width")
    if residual is not None and (tuple(residual.shape) != (n, cout)
                                 or residual.dtype != features.dtype
                                 or not residual.is_contiguous()):
        raise ValueError(f"residual must be a contiguous ({n}, {cout}) {features.dtype} tensor")
    lib = N.load()
    ws = N.workspace(256, dev)
    rc = lib.sv_conv3d_forward_dd(
        features.data_ptr(), n, cin, neighbors.data_ptr(), neighbors.shape[1],
        plan.buffer.data_ptr(), plan.nbytes, weight_oki.data_ptr(), N.ptr(bias),
        N.ptr(residual), cout, N.DTYPE_CODE[features.dtype], out.data_ptr(), ws.data_ptr(), 256,
        N.status_word(dev).data_ptr(), N.stream(dev))
    N.check(rc, "sparse_conv3d (deduplicated tiles)")
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


def conv3d_forward_halo(features, neighbors, weight, bias, cout, rows, tile_order, halo_from,
                        flags, flag_count, epoch, *, out, residual=None) -> torch.Tensor:
    """``sv_conv3d_forward_halo``: one tcgen05 launch over ``rows`` whose tiles from tile-order
    position ``halo_from`` on wait, inside the kernel, for ``flag_count`` peer flags (a ctypes
    array of device pointers) to reach ``epoch``."""

    n, cin = features.shape
    dev = features.device
    lib = N.load()
    ws = N.workspace(256, dev)
    rc = lib.sv_conv3d_forward_halo(
        features.data_ptr(), n, cin, neighbors.data_ptr(), neighbors.shape[1], rows.data_ptr(),
        rows.numel(), N.ptr(tile_order), int(halo_from), flags, int(flag_count), int(epoch),
        weight.data_ptr(), N.ptr(bias), N.ptr(residual), cout, N.DTYPE_CODE[features.dtype],
        out.data_ptr(), ws.data_ptr(), 256, N.status_word(dev).data_ptr(), N.stream(dev),
    )
    N.check(rc, "sparse_conv3d (halo)")
    return out


# ---- backward --------------------------------------------------------------------------------


def kmap_pairs(neighbors: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per-offset pair lists of a kernel map: ``(offsets [K+1], src [P], dst [P])`` with
    ``src = nbr[dst, k]`` for the pairs of offset k in ``offsets[k]:offsets[k+1]``, destinations
    ascending (``sv_kmap_pairs_count`` / ``sv_kmap_pairs_emit``; one host synchronisation)."""

    N.require_cuda(neighbors, "neighbors")
    nbr = neighbors.contiguous()
    n, kvol = nbr.shape
    dev = nbr.device
    lib = N.load()
    ws_bytes = lib.sv_kmap_pairs_workspace_bytes(n, kvol)
    ws = N.workspace(ws_bytes, dev)
    status = N.status_word(dev)
    total = ctypes.c_int64(0)
    rc = lib.sv_kmap_pairs_count(nbr.data_ptr(), n, kvol, ctypes.byref(total), ws.data_ptr(),
                                 ws_bytes, status.data_ptr(), N.stream(dev))
    N.check(rc, "kmap_pairs")
    p = int(total.value)
    offsets = torch.empty(kvol + 1, dtype=torch.int32, device=dev)
    src = torch.empty(max(p, 1), dtype=torch.int32, device=dev)
    dst = torch.empty(max(p, 1), dtype=torch.int32, device=dev)
    rc = lib.sv_kmap_pairs_emit(nbr.data_ptr(), n, kvol, offsets.data_ptr(), src.data_ptr(),
                                dst.data_ptr(), p, ws.data_ptr(), ws_bytes, status.data_ptr(),
                                N.stream(dev))
    N.check(rc, "kmap_pairs")
    return offsets, src[:p], dst[:p]


def weight_flip_transpose(weight: torch.Tensor) -> torch.Tensor:
    """``W'[i, j, o] = W[o, K-1-j, i]`` for a spconv ``(O, kD, kH, kW, I)`` weight, returned as
    ``(I, kD, kH, kW, O)``: the weight of the forward convolution that computes the input
    gradient (``sv_weight_flip_transpose``)."""

    N.require_cuda(weight, "weight")
    w = weight.contiguous()
    o, kd, kh, kw, i = w.shape
    out = torch.empty((i, kd, kh, kw, o), dtype=w.dtype, device=w.device)
    rc = N.load().sv_weight_flip_transpose(w.data_ptr(), o, kd * kh * kw, i,
                                           N.DTYPE_CODE[w.dtype], out.data_ptr(),
                                           N.stream(w.device))
    N.check(rc, "weight_flip_transpose")
    return out


def conv3d_wgrad(features: torch.Tensor, dout: torch.Tensor,
                 pairs: tuple[torch.Tensor, torch.Tensor, torch.Tensor], kernel_shape,
                 *, algo: int = N.SV_CONV_AUTO) -> torch.Tensor:
    """Weight gradient in spconv layout ``(Cout, kD, kH, kW, Cin)`` (``sv_conv3d_wgrad``)."""

    offsets, src, dst = pairs
    f = features.contiguous()
    g = dout.contiguous().to(f.dtype)
    cin, cout = f.shape[1], g.shape[1]
    kvol = offsets.numel() - 1
    dev = f.device
    out = torch.empty((cout, *kernel_shape, cin), dtype=f.dtype, device=dev)
    lib = N.load()
    code = N.DTYPE_CODE[f.dtype]
    ws_bytes = lib.sv_conv3d_wgrad_workspace_bytes(cin, cout, kvol, code, algo)
    ws = N.workspace(ws_bytes, dev) if ws_bytes else None
    rc = lib.sv_conv3d_wgrad(f.data_ptr(), g.data_ptr(), cin, cout, kvol, offsets.data_ptr(),
                             src.data_ptr(), dst.data_ptr(), code, out.data_ptr(), algo,
                             N.ptr(ws), ws_bytes, N.status_word(dev).data_ptr(), N.stream(dev))
    N.check(rc, "conv3d_wgrad")
    return out


def conv3d_dbias(dout: torch.Tensor) -> torch.Tensor:
    """Column sums of ``dout`` in a fixed order (``sv_conv3d_dbias``)."""

    g = dout.contiguous()
    n, c = g.shape
    dev = g.device
    out = torch.empty(c, dtype=g.dtype, device=dev)
    lib = N.load()
    ws_bytes = lib.sv_conv3d_dbias_workspace_bytes(n, c)
    ws = N.workspace(ws_bytes, dev)
    rc = lib.sv_conv3d_dbias(g.data_ptr(), n, c, N.DTYPE_CODE[g.dtype], out.data_ptr(),
                             ws.data_ptr(), ws_bytes, N.stream(dev))
    N.check(rc, "conv3d_dbias")
    return out


def conv3d_dgrad(dout: torch.Tensor, neighbors: torch.Tensor, weight: torch.Tensor, *,
                 unique: bool, row_order=None, tile_order=None,
                 algo: int = N.SV_CONV_AUTO) -> torch.Tensor:
    """Input gradient: the forward convolution of ``dout`` over the same map with the
    flipped, transposed weight. With duplicate coordinates (``unique=False``) the gradient
    flows only into the row each coordinate resolves to (the largest duplicate): ``dout`` is
    first summed into that row, and the other duplicates get zero."""

    w_t = weight_flip_transpose(weight)
    cin = weight.shape[-1]
    g = dout.contiguous().to(weight.dtype)
    n, kvol = neighbors.shape
    center = kvol // 2
    if not unique:
        resolved = neighbors[:, center].long()
        merged = torch.zeros(g.shape, dtype=torch.float32, device=g.device)
        merged.index_add_(0, resolved, g.float())
        g = merged.to(g.dtype)
    dx = conv3d_forward(g, neighbors, w_t, N.SV_WEIGHT_OKI, None, cin, row_order=row_order,
                        tile_order=tile_order, algo=algo)
    if not unique:
        own = resolved == torch.arange(n, device=g.device)
        dx = dx * own[:, None].to(dx.dtype)
    return dx


class SparseConv3DFunction(torch.autograd.Function):
    """Submanifold conv with the gradients of mlx_diffuser's fallback
    (``src/mlx_diffuser/kernels/sparse.py:39-55``): input gradient through the transposed map,
    weight gradient per offset from the pair lists, bias gradient as column sums."""

    @staticmethod
    def forward(ctx, features, weight, bias, neighbors, topology, algo):
        row_order, tile_order = topology.schedule()
        out = conv3d_forward(features.contiguous(), neighbors, weight.contiguous(),
                             N.SV_WEIGHT_OKI, bias, weight.shape[0], row_order=row_order,
                             tile_order=tile_order, algo=algo)
        ctx.save_for_backward(features, weight)
        ctx.neighbors = neighbors
        ctx.topology = topology
        ctx.algo = algo
        ctx.has_bias = bias is not None
        return out

    @staticmethod
    def backward(ctx, dout):
        features, weight = ctx.saved_tensors
        topo = ctx.topology
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            row_order, tile_order = topo.schedule()
            dx = conv3d_dgrad(dout, ctx.neighbors, weight, unique=topo.unique(),
                              row_order=row_order, tile_order=tile_order, algo=ctx.algo)
        if ctx.needs_input_grad[1]:
            dw = conv3d_wgrad(features, dout, topo.pairs(), weight.shape[1:4], algo=ctx.algo)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = conv3d_dbias(dout.to(weight.dtype))
        return dx, dw, db, None, None, None
