"""CPU oracle for the TRELLIS sparse-voxel path -- TEST INFRASTRUCTURE ONLY.

This is a NumPy restatement of mlx_diffuser's sparse-voxel hot path. It is the checker for
the CUDA library, never part of it: only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import it. Every function cites the reference lines it
restates (paths relative to the mlx_diffuser project root).

It is pinned against the reference itself: ``tests/golden/make_golden.py`` runs the reference's
own ``src/mlx_diffuser/layers/sparse.py`` and ``src/mlx_diffuser/kernels/sparse.py`` unmodified
under a NumPy stand-in for MLX and commits the outputs as fixtures; ``tests/test_oracle.py``
checks this module against them bit-exactly (integers) and to float32 rounding (features).
"""

from __future__ import annotations

import math

import numpy as np

# --------------------------------------------------------------------------------------------
# kernel map
# --------------------------------------------------------------------------------------------


def _triple(value) -> tuple[int, int, int]:
    if isinstance(value, (int, np.integer)):
        return (int(value), int(value), int(value))
    value = tuple(int(v) for v in value)
    if len(value) != 3:
        raise ValueError("sparse submanifold kernels must have three odd dimensions")
    return value  # type: ignore[return-value]


def kernel_offsets(kernel_size, dilation=1) -> list[tuple[int, int, int]]:
    """Offsets in the reference's order (``src/mlx_diffuser/layers/sparse.py:153-169``).

    The outer loop runs over the first spatial column (coords column 1); offset ``k`` adds
    ``(d1, d2, d3)`` to coords columns 1, 2, 3.
    """

    kernel = _triple(kernel_size)
    dil = _triple(dilation)
    if any(k % 2 == 0 for k in kernel):
        raise ValueError("sparse submanifold kernels must have three odd dimensions")
    return [
        (
            (a - kernel[0] // 2) * dil[0],
            (b - kernel[1] // 2) * dil[1],
            (c - kernel[2] // 2) * dil[2],
        )
        for a in range(kernel[0])
        for b in range(kernel[1])
        for c in range(kernel[2])
    ]


def build_neighbor_map_dict(coords, kernel_size, dilation=1) -> np.ndarray:
    """Literal restatement of ``build_neighbor_map`` (``src/mlx_diffuser/layers/sparse.py:146-175``).

    A dict from the 4-tuple ``(b, c1, c2, c3)`` to the row index; a later duplicate row
    overwrites an earlier one (``:159``); a missing neighbour is ``-1`` (``:170-174``).
    Pure-Python loops: used for small cases and as the faithful CPU baseline.
    """

    offsets = kernel_offsets(kernel_size, dilation)
    host = np.asarray(coords, dtype=np.int32)
    lookup = {tuple(int(v) for v in row): i for i, row in enumerate(host)}
    out = np.full((len(host), len(offsets)), -1, dtype=np.int32)
    for p, row in enumerate(host):
        b, c1, c2, c3 = (int(v) for v in row)
        for k, (d1, d2, d3) in enumerate(offsets):
            out[p, k] = lookup.get((b, c1 + d1, c2 + d2, c3 + d3), -1)
    return out


_SPATIAL_BITS = 20  # packed key: each spatial column 20 bits (signed, biased), batch 4 bits


def build_neighbor_map(coords, kernel_size, dilation=1) -> np.ndarray:
    """Vectorised, bit-exact equivalent of :func:`build_neighbor_map_dict`.

    Rows are packed into one 64-bit key when every coordinate, shifted by the largest offset,
    fits in 20 signed bits and the batch index in the remaining 4 bits ([0, 16)); otherwise the
    dict version runs.
    Duplicate rows resolve to the largest row index, which is what the reference's dict
    comprehension keeps (``src/mlx_diffuser/layers/sparse.py:159``).
    """

    offsets = kernel_offsets(kernel_size, dilation)
    host = np.asarray(coords, dtype=np.int32).reshape(-1, 4)
    n = len(host)
    if n == 0:
        return np.zeros((0, len(offsets)), dtype=np.int32)
    reach = max(abs(v) for off in offsets for v in off)
    lim = (1 << (_SPATIAL_BITS - 1)) - 1 - reach
    spatial = host[:, 1:].astype(np.int64)
    if (
        host[:, 0].min() < 0
        or host[:, 0].max() >= (1 << (64 - 3 * _SPATIAL_BITS))
        or spatial.min() < -lim
        or spatial.max() > lim
    ):
        return build_neighbor_map_dict(host, kernel_size, dilation)

    bias = 1 << (_SPATIAL_BITS - 1)

    def pack(b, c1, c2, c3):
        return (
            (b << (3 * _SPATIAL_BITS))
            | ((c1 + bias) << (2 * _SPATIAL_BITS))
            | ((c2 + bias) << _SPATIAL_BITS)
            | (c3 + bias)
        )

    b = host[:, 0].astype(np.int64)
    keys = pack(b, spatial[:, 0], spatial[:, 1], spatial[:, 2])
    # last occurrence of every key == largest row index among duplicates
    rev_keys, rev_first = np.unique(keys[::-1], return_index=True)
    rows = (n - 1 - rev_first).astype(np.int32)
    out = np.full((n, len(offsets)), -1, dtype=np.int32)
    for k, (d1, d2, d3) in enumerate(offsets):
        q = pack(b, spatial[:, 0] + d1, spatial[:, 1] + d2, spatial[:, 2] + d3)
        pos = np.searchsorted(rev_keys, q)
        pos = np.minimum(pos, len(rev_keys) - 1)
        hit = rev_keys[pos] == q
        out[hit, k] = rows[pos[hit]]
    return out


# --------------------------------------------------------------------------------------------
# convolution
# --------------------------------------------------------------------------------------------


def spconv_weight_to_kio(weight: np.ndarray) -> np.ndarray:
    """``(O, kD, kH, kW, I) -> (kD*kH*kW, I, O)`` as ``SparseConv3D.__call__`` does
    (``src/mlx_diffuser/layers/sparse.py:224-226``)."""

    w = np.asarray(weight)
    o, kd, kh, kw, i = w.shape
    return np.ascontiguousarray(w.transpose(1, 2, 3, 4, 0).reshape(kd * kh * kw, i, o))


def sparse_conv3d(features, neighbors, weights, bias, *, accum=np.float32) -> np.ndarray:
    """Gather-matmul-accumulate fallback (``src/mlx_diffuser/kernels/sparse.py:39-55``).

    ``out = bias + sum_k (features[max(nbr[:,k],0)] @ W[k]) * (nbr[:,k] >= 0)``, evaluated in
    ``accum`` (float32 like the reference run in float32, or float64 for tie-breaks). The
    shape checks follow ``sparse_conv3d`` (``src/mlx_diffuser/kernels/sparse.py:78-88``).
    """

    f = np.asarray(features).astype(accum)
    nbr = np.asarray(neighbors).astype(np.int32)
    w = np.asarray(weights).astype(accum)
    b = np.asarray(bias).astype(accum)
    if f.ndim != 2:
        raise ValueError(f"features must be 2D, got {f.shape}")
    if nbr.ndim != 2 or nbr.shape[0] != f.shape[0]:
        raise ValueError("neighbors must have shape (N, kernel_volume)")
    if w.ndim != 3 or w.shape[:2] != (nbr.shape[1], f.shape[1]):
        raise ValueError(
            f"weights must have shape ({nbr.shape[1]}, {f.shape[1]}, Cout), got {w.shape}"
        )
    if b.shape != (w.shape[2],):
        raise ValueError(f"bias must have shape ({w.shape[2]},), got {b.shape}")
    out = np.broadcast_to(b, (f.shape[0], b.shape[0])).copy()
    for k in range(nbr.shape[1]):
        index = nbr[:, k]
        valid = index >= 0
        if not valid.any():
            continue
        out[valid] += f[index[valid]] @ w[k]
    return out


# --------------------------------------------------------------------------------------------
# pooling
# --------------------------------------------------------------------------------------------


def downsample_coords(coords, factor: int = 2) -> tuple[np.ndarray, np.ndarray]:
    """Coordinates and inverse of ``sparse_downsample`` (``src/mlx_diffuser/layers/sparse.py:250-253``).

    Spatial columns are floor-divided by ``factor``; rows are made unique in lexicographic
    (signed) order with ``np.unique(axis=0)``; the inverse maps every fine row to its coarse row.
    """

    if factor < 1:
        raise ValueError("factor must be positive")
    host = np.asarray(coords, dtype=np.int32).reshape(-1, 4).copy()
    host[:, 1:] //= factor
    if len(host) == 0:
        return np.zeros((0, 4), np.int32), np.zeros((0,), np.int32)
    new_coords, inverse = np.unique(host, axis=0, return_inverse=True)
    return new_coords.astype(np.int32), np.asarray(inverse).reshape(-1).astype(np.int32)


def downsample_features(features, inverse, num_out: int, *, accum=np.float32) -> np.ndarray:
    """``summed / (count + 1)`` pooling of ``sparse_downsample``
    (``src/mlx_diffuser/layers/sparse.py:254-266``): scatter-add of the features and of ones,
    then a divide by ``count + 1`` (the zero-initialised ``include_self`` mean)."""

    f = np.asarray(features).astype(accum)
    inv = np.asarray(inverse, dtype=np.int64)
    count = np.zeros((num_out, 1), dtype=np.float32)
    np.add.at(count, inv, np.float32(1.0))
    summed = np.zeros((num_out, f.shape[1]), dtype=accum)
    np.add.at(summed, inv, f)
    return summed / (count + 1).astype(accum)


def downsample_spatial_shape(spatial_shape, factor: int) -> tuple[int, int, int]:
    """``ceil(s / factor)`` per axis (``src/mlx_diffuser/layers/sparse.py:269-274``)."""

    s = spatial_shape or (0, 0, 0)
    return (math.ceil(s[0] / factor), math.ceil(s[1] / factor), math.ceil(s[2] / factor))


def upsample_features(features, inverse) -> np.ndarray:
    """Nearest gather of ``sparse_upsample`` (``src/mlx_diffuser/layers/sparse.py:295``)."""

    return np.asarray(features)[np.asarray(inverse, dtype=np.int64)]


def valid_pairs(neighbors) -> int:
    """P: the number of valid (output, input, offset) triples in a kernel map."""

    return int((np.asarray(neighbors) >= 0).sum())


def sparse_conv3d_fallback_literal(features, neighbors, weights, bias) -> np.ndarray:
    """Operation-for-operation copy of the reference's fallback loop
    (``src/mlx_diffuser/kernels/sparse.py:47-55``) in NumPy float32: every offset gathers all
    N rows through ``max(index, 0)``, multiplies by W[k] and masks the invalid rows. Same result
    as :func:`sparse_conv3d`, same amount of work as the reference; the CPU baseline times it."""

    f = np.asarray(features, np.float32)
    nbr = np.asarray(neighbors, np.int32)
    w = np.asarray(weights, np.float32)
    b = np.asarray(bias, np.float32)
    points, kernel_volume = nbr.shape
    out = np.broadcast_to(b, (points, b.shape[0]))
    for k in range(kernel_volume):
        index = nbr[:, k]
        valid = index >= 0
        safe_index = np.maximum(index, 0)
        contribution = f[safe_index] @ w[k]
        out = out + contribution * valid[:, None]
    return out


# --------------------------------------------------------------------------------------------
# topology: subdivision, attention windows, occupancy -> coordinates
# --------------------------------------------------------------------------------------------


def subdivide(coords, features) -> tuple[np.ndarray, np.ndarray]:
    """``sparse_subdivide`` (``src/mlx_diffuser/layers/sparse.py:298-318``): row i becomes rows
    8i + j, j = 4z + 2y + x in the nested order of the reference's offset list, at
    (b, 2*c1 + z, 2*c2 + y, 2*c3 + x), each with a copy of feature row i."""

    coords = np.asarray(coords, np.int32)
    n = len(coords)
    child = np.array([[0, z, y, x] for z in range(2) for y in range(2) for x in range(2)],
                     np.int32)
    scaled = coords[:, None, :] * np.array([1, 2, 2, 2], np.int32)
    out_coords = (scaled + child[None]).reshape(n * 8, 4)
    features = np.asarray(features)
    out_features = np.repeat(features, 8, axis=0)
    return out_coords, out_features


def attention_groups(coords, window_size, shift_window=(0, 0, 0)) -> list[np.ndarray]:
    """``_attention_groups`` (``src/mlx_diffuser/layers/sparse.py:321-342``): rows grouped by
    (b) or by (b, (xyz + shift) // window); groups in the order their first row appears, rows
    ascending inside a group (a dict of lists filled in row order)."""

    coords = np.asarray(coords, np.int32)
    if window_size is None:
        keys = coords[:, :1]
    else:
        shift = np.asarray(shift_window, dtype=np.int32)
        keys = np.concatenate([coords[:, :1], (coords[:, 1:] + shift) // window_size], axis=1)
    groups: dict[tuple[int, ...], list[int]] = {}
    for index, key in enumerate(keys):
        groups.setdefault(tuple(int(v) for v in key), []).append(index)
    return [np.asarray(rows, dtype=np.int32) for rows in groups.values()]


def occupied_coordinates(logits, threshold: float = 0.0, dtype: str = "float32") -> np.ndarray:
    """The ``np.argwhere(logits > threshold)`` step of ``occupied_coordinates``
    (``src/mlx_diffuser/models/trellis.py:278-285``) on a [B, D, H, W] grid whose values are
    exact in ``dtype`` ("float32", "float16" or "bfloat16"; given as float32 arrays). The
    threshold is rounded to float32 and then to ``dtype``, as MLX's promotion of a Python float
    scalar does, and the comparison of two values exact in ``dtype`` is made in float32."""

    logits = np.asarray(logits, np.float32)
    thr = np.float32(threshold)
    if dtype == "float16":
        thr = np.float32(np.float16(thr))
    elif dtype == "bfloat16":
        thr = round_to_bf16(np.array([thr], np.float32))[0]
    return np.argwhere(logits > thr).astype(np.int32)


def round_to_bf16(values) -> np.ndarray:
    """float32 values rounded to the nearest bfloat16 (ties to even), returned as float32."""

    v = np.ascontiguousarray(np.asarray(values, np.float32))
    bits = v.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(v), v, out)


# --------------------------------------------------------------------------------------------
# residual block around the convolutions
# --------------------------------------------------------------------------------------------


def layernorm32(h, weight=None, bias=None, eps: float = 1e-6) -> np.ndarray:
    """``LayerNorm32`` (``src/mlx_diffuser/layers/trellis.py:16-43``) in float32."""

    h = np.asarray(h, np.float32)
    mean = h.mean(-1, keepdims=True)
    var = np.square(h - mean).mean(-1, keepdims=True)
    h = (h - mean) / np.sqrt(var + np.float32(eps))
    if weight is not None:
        h = h * weight + bias
    return h.astype(np.float32)


def silu(h) -> np.ndarray:
    h = np.asarray(h, np.float32)
    return (h / (1.0 + np.exp(-h))).astype(np.float32)


def resblock(coords, feats, emb, p: dict, *, nbr=None) -> np.ndarray:
    """``_SparseResBlock3D.__call__`` after its optional resampling
    (``src/mlx_diffuser/models/trellis_slat.py:71-82``), float32: ``p`` holds norm1_w/_b,
    conv1_w/_b, conv2_w/_b (spconv layout), emb_w/_b and optionally skip_w/_b. The modulation
    rows are picked by the batch column when ``emb`` has one row per batch element."""

    coords = np.asarray(coords, np.int32)
    if nbr is None:
        nbr = build_neighbor_map(coords, 3)
    proj = silu(emb) @ p["emb_w"].T + p["emb_b"]
    scale, shift = np.split(proj.astype(np.float32), 2, axis=-1)
    batch_size = int(coords[:, 0].max()) + 1 if len(coords) else 0
    if scale.shape[0] == batch_size:
        scale, shift = scale[coords[:, 0]], shift[coords[:, 0]]
    a = silu(layernorm32(feats, p["norm1_w"], p["norm1_b"]))
    h = sparse_conv3d(a, nbr, spconv_weight_to_kio(p["conv1_w"]), p["conv1_b"])
    h = layernorm32(h) * (1 + scale) + shift
    h = sparse_conv3d(silu(h), nbr, spconv_weight_to_kio(p["conv2_w"]), p["conv2_b"])
    skip = feats @ p["skip_w"].T + p["skip_b"] if "skip_w" in p else feats
    return (h + skip).astype(np.float32)


# --------------------------------------------------------------------------------------------
# gradients
# --------------------------------------------------------------------------------------------


def sparse_conv3d_grads(features, neighbors, weights, dout, *, accum=np.float32):
    """Gradients of the fallback (``src/mlx_diffuser/kernels/sparse.py:39-55``) with respect to
    features, the (K, Cin, Cout) weights and the bias, for an output gradient ``dout``:
    d features[q] = sum over (p, k) with nbr[p, k] == q of dout[p] @ W[k]^T;
    d W[k] = features[nbr[valid, k]]^T @ dout[valid]; d bias = sum over rows of dout."""

    features = np.asarray(features, accum)
    dout = np.asarray(dout, accum)
    w = np.asarray(weights, accum)
    nbr = np.asarray(neighbors)
    dx = np.zeros_like(features)
    dw = np.zeros_like(w)
    for k in range(nbr.shape[1]):
        valid = nbr[:, k] >= 0
        src = nbr[valid, k]
        np.add.at(dx, src, dout[valid] @ w[k].T)
        dw[k] = features[src].T @ dout[valid]
    return dx, dw, dout.sum(0)
