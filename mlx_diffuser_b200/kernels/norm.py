"""Binding of ``sv_rownorm``: LayerNorm32 with the residual block's modulation and SiLU fused
into one pass over the rows (``src/mlx_diffuser/layers/trellis.py:16-43``,
``src/mlx_diffuser/models/trellis_slat.py:77-80``)."""

from __future__ import annotations

import torch

from .. import _native as N


def row_norm(
    x: torch.Tensor,
    *,
    weight: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    scale: torch.Tensor | None = None,
    shift: torch.Tensor | None = None,
    coords: torch.Tensor | None = None,
    batch_size: int | None = None,
    silu: bool = False,
    eps: float = 1e-6,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``silu?( LN32(x) [* weight + bias] [* (1 + scale[b]) + shift[b]] )`` over the last axis,
    fp32 inside, one rounding to ``x.dtype``. ``weight`` / ``bias``: fp32 ``[C]``. ``scale`` /
    ``shift``: ``[B, C]`` (or ``[C]`` / ``[1, C]``, shared by every row), rows picked by
    ``coords[:, 0]`` of an ``[N, 4]`` int32 coordinate tensor."""

    N.require_cuda(x, "x")
    c = x.shape[-1]
    flat = x.reshape(-1, c).contiguous()
    n = flat.shape[0]
    if flat.dtype not in N.DTYPE_CODE:
        raise ValueError(f"row_norm: unsupported dtype {flat.dtype}")
    dev = flat.device
    if weight is not None:
        weight = weight.to(device=dev, dtype=torch.float32).contiguous()
        if weight.shape != (c,):
            raise ValueError(f"row_norm: weight must have shape ({c},)")
    if bias is not None:
        bias = bias.to(device=dev, dtype=torch.float32).contiguous()
    mods: list[torch.Tensor | None] = []
    for name, t in (("scale", scale), ("shift", shift)):
        if t is None:
            mods.append(None)
            continue
        t = t.to(device=dev, dtype=flat.dtype)
        if t.ndim == 1:
            t = t[None]
        if t.ndim != 2 or t.shape[1] != c:
            raise ValueError(f"row_norm: {name} must have shape (B, {c})")
        if t.stride(1) != 1 or (t.shape[0] > 1 and t.stride(0) < c):
            t = t.contiguous()
        mods.append(t)
    live = [m for m in mods if m is not None]
    b = 0
    mod_stride = 0
    if live:
        if coords is None:
            raise ValueError("row_norm: modulation needs the coordinates (batch column)")
        rows = {m.shape[0] for m in live}
        b = int(batch_size) if batch_size is not None else max(rows)
        if any(r not in (1, b) for r in rows):
            raise ValueError(f"row_norm: modulation rows {sorted(rows)} for batch {b}")
        strides = {0 if m.shape[0] == 1 else m.stride(0) for m in live}
        if len(strides) > 1:  # scale and shift laid out differently: make both dense
            mods = [None if m is None else m.expand(b, c).contiguous() for m in mods]
            strides = {c}
        mod_stride = strides.pop()
        coords = coords.to(device=dev, dtype=torch.int32).contiguous()
        if coords.shape != (n, 4):
            raise ValueError(f"row_norm: coords must have shape ({n}, 4)")
    if out is None:
        out = torch.empty_like(flat)
    rc = N.load().sv_rownorm(
        flat.data_ptr(), n, c, N.DTYPE_CODE[flat.dtype], float(eps), N.ptr(weight), N.ptr(bias),
        N.ptr(mods[0]), N.ptr(mods[1]), mod_stride, N.ptr(coords), b, int(bool(silu)),
        out.data_ptr(),
        N.status_word(dev).data_ptr(), N.stream(dev),
    )
    N.check(rc, "row_norm")
    return out.reshape(x.shape)
