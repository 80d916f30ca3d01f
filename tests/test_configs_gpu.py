"""The benchmark configurations at their stated sizes, against the fp32 oracle.

* config 1: 64^3 noisy shell (~20k voxels), conv 128 -> 128 in fp32 (rtol 1e-4);
* config 3: SLat-flow-style I/O stack in fp16, batch 2 (ResBlock 8 -> 128 with a 1x1 skip,
  downsample, conv 128 -> 1024, upsample, convs 1024 -> 128 -> 8), max relative error 1e-2;
* config 4: 128^3 union of six shells (~237k voxels), convs 64 -> 64 -> 32 in bf16;
* config 5: uniform and surface-shell occupancy 0.5 / 2 / 8 / 30 % on 64^3 and 128^3, batch 16,
  widths 32 / 128 / 512 / 1024 in bf16 (kernel maps bit-exact; convs on sampled rows against the
  oracle and on every row through random projections).

For the fp16/bf16 cases the reference is computed in fp32 from the same rounded inputs and
weights; "max relative error" is max|out - ref| / max|ref|.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mlx_diffuser_b200 import _native as N
from mlx_diffuser_b200 import scenes
from mlx_diffuser_b200.layers.sparse import (
    SparseConv3D,
    SparseTensor,
    build_neighbor_map,
    sparse_downsample,
    sparse_upsample,
)
from oracle import sparse_oracle as O
from tests.fullsize import device_features, oracle_rows, projection_error

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def max_rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def _rounded(a, dtype):
    return torch.from_numpy(np.asarray(a, np.float32)).to(dtype).float().numpy()


def _conv(cin, cout, weight, bias, dtype):
    conv = SparseConv3D(cin, cout, 3).to(DEV)
    conv.conv.weight = torch.from_numpy(weight).to(DEV, dtype)
    conv.conv.bias = torch.from_numpy(bias).to(DEV, dtype)
    return conv


def test_config1_fp32_shell64_conv128():
    coords = scenes.shell64(0)
    f = scenes.normal_features(len(coords), 128, seed=1)
    w = (np.random.default_rng(2).standard_normal((128, 3, 3, 3, 128)) / np.sqrt(27 * 128)).astype(np.float32)
    b = np.zeros(128, np.float32)
    x = SparseTensor(torch.from_numpy(f).to(DEV), torch.from_numpy(coords).to(DEV))
    out = _conv(128, 128, w, b, torch.float32)(x).features.cpu().numpy()
    nbr = O.build_neighbor_map(coords, 3)
    assert np.array_equal(x.cache["neighbors_3_1_(1, 1, 1)"].cpu().numpy(), nbr)
    ref = O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w), b, accum=np.float64)
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
    N.check_device_status(DEV)


# ---- config 3 -------------------------------------------------------------------------------


def _layernorm32(h, weight=None, bias=None, eps=1e-6):
    """LayerNorm32 of the reference (src/mlx_diffuser/layers/trellis.py:16-43) in fp32."""

    h = np.asarray(h, np.float32)
    mean = h.mean(-1, keepdims=True)
    var = ((h - mean) ** 2).mean(-1, keepdims=True)
    h = (h - mean) / np.sqrt(var + eps)
    if weight is not None:
        h = h * weight + bias
    return h


def _silu(h):
    return h / (1.0 + np.exp(-h))


def _torch_ln32(h, weight=None, bias=None, eps=1e-6):
    dtype = h.dtype
    h = h.float()
    h = torch.nn.functional.layer_norm(h, (h.shape[-1],), weight, bias, eps)
    return h.to(dtype)


def test_config3_slat_io_stack_fp16():
    """ResBlock pattern of src/mlx_diffuser/models/trellis_slat.py:71-82 around the sparse ops:
    SiLU(LN32) -> conv 8->128 -> LN32 * (1 + scale) + shift -> SiLU -> conv 128->128, plus a
    1x1 skip; then downsample -> conv 128->1024 -> upsample -> conv 1024->128 -> conv 128->8."""

    dtype = torch.float16
    rng = np.random.default_rng(30)
    coords = scenes.batched([scenes.shell64(3), scenes.shell64(4)])
    n = len(coords)
    x0 = _rounded(scenes.normal_features(n, 8, seed=31), dtype)
    ws = {
        "c1": _rounded(scenes.conv_weight(128, 8, 3, 32), dtype),
        "c2": _rounded(scenes.conv_weight(128, 128, 3, 33), dtype),
        "c3": _rounded(scenes.conv_weight(1024, 128, 3, 34), dtype),
        "c4": _rounded(scenes.conv_weight(128, 1024, 3, 35), dtype),
        "c5": _rounded(scenes.conv_weight(8, 128, 3, 36), dtype),
    }
    bs = {k: _rounded(rng.standard_normal(w.shape[0]) * 0.05, dtype) for k, w in ws.items()}
    skip_w = _rounded(rng.standard_normal((128, 8)) / np.sqrt(8), dtype)
    skip_b = _rounded(rng.standard_normal(128) * 0.05, dtype)
    scale = _rounded(rng.standard_normal((2, 128)) * 0.1, dtype)
    shift = _rounded(rng.standard_normal((2, 128)) * 0.1, dtype)

    # ---- GPU path: the library's sparse ops, torch for the dense glue ----
    convs = {k: _conv(w.shape[-1], w.shape[0], w, bs[k], dtype) for k, w in ws.items()}
    t = lambda a: torch.from_numpy(np.asarray(a)).to(DEV, dtype)  # noqa: E731
    x = SparseTensor(t(x0), torch.from_numpy(coords).to(DEV))
    b_idx = x.coords[:, 0].long()
    h = x.replace(torch.nn.functional.silu(_torch_ln32(x.features)))
    h = convs["c1"](h)
    h = h.replace(_torch_ln32(h.features) * (1 + t(scale)[b_idx]) + t(shift)[b_idx])
    h = convs["c2"](h.replace(torch.nn.functional.silu(h.features)))
    h = h + (x.features @ t(skip_w).T + t(skip_b))
    d = sparse_downsample(h, 2)
    d = convs["c3"](d)
    u = sparse_upsample(d, 2)
    u = convs["c4"](u)
    y = convs["c5"](u).features.float().cpu().numpy()
    N.check_device_status(DEV)

    # ---- fp32 oracle on the same rounded inputs ----
    nbr = O.build_neighbor_map(coords, 3)
    conv = lambda f, k, nb: O.sparse_conv3d(f, nb, O.spconv_weight_to_kio(ws[k]), bs[k])  # noqa: E731
    bi = coords[:, 0]
    r = _silu(_layernorm32(x0))
    r = conv(r, "c1", nbr)
    r = _layernorm32(r) * (1 + scale[bi]) + shift[bi]
    r = conv(_silu(r), "c2", nbr)
    r = r + (x0 @ skip_w.T + skip_b)
    dc, inv = O.downsample_coords(coords, 2)
    assert np.array_equal(d.coords.cpu().numpy(), dc)
    r = O.downsample_features(r, inv, len(dc))
    r = conv(r, "c3", O.build_neighbor_map(dc, 3))
    r = O.upsample_features(r, inv)
    r = conv(r, "c4", nbr)
    r = conv(r, "c5", nbr)
    assert max_rel_err(y, r) <= 1e-2


# ---- config 4 -------------------------------------------------------------------------------


def test_config4_scene128_convs_64_64_32_bf16():
    """Both layers against the fp32 oracle: layer 1 on its own, and the two-layer chain against
    the oracle's fp32 chain from the original inputs (the GPU rounds the 64-channel intermediate
    to bf16; the oracle does not), so the two-layer error growth is measured too."""

    dtype = torch.bfloat16
    coords = scenes.scene128(0)
    f = _rounded(scenes.normal_features(len(coords), 64, seed=40), dtype)
    w1 = _rounded(scenes.conv_weight(64, 64, 3, 41), dtype)
    w2 = _rounded(scenes.conv_weight(32, 64, 3, 42), dtype)
    z64, z32 = np.zeros(64, np.float32), np.zeros(32, np.float32)
    x = SparseTensor(torch.from_numpy(f).to(DEV, dtype), torch.from_numpy(coords).to(DEV))
    h = _conv(64, 64, w1, z64, dtype)(x)
    y = _conv(64, 32, w2, z32, dtype)(h)
    N.check_device_status(DEV)
    nbr = O.build_neighbor_map(coords, 3)
    assert np.array_equal(x.cache["neighbors_3_1_(1, 1, 1)"].cpu().numpy(), nbr)
    r1 = O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w1), z64)
    assert max_rel_err(h.features.float().cpu().numpy(), r1) <= 1e-2
    # the chain: layer 2 of the oracle consumes the oracle's own fp32 layer-1 output
    r2 = O.sparse_conv3d(r1, nbr, O.spconv_weight_to_kio(w2), z32)
    assert max_rel_err(y.features.float().cpu().numpy(), r2) <= 1e-2


# ---- config 5 -------------------------------------------------------------------------------

CONFIG5_WIDTHS = (32, 128, 512, 1024)
SAMPLED_ROWS = 1024


def config5_coords(layout: str, grid: int, occupancy: float) -> np.ndarray:
    """16 independently seeded elements of one sweep cell."""

    if layout == "uniform":
        return scenes.batched([scenes.uniform(grid, occupancy, 900 + b) for b in range(16)])
    return scenes.batched([scenes.shell_fraction(grid, occupancy, 950 + b) for b in range(16)])


@pytest.mark.parametrize("layout", ["uniform", "shell"])
@pytest.mark.parametrize("grid", [64, 128])
@pytest.mark.parametrize("occupancy", [0.005, 0.02, 0.08, 0.30])
def test_config5_sweep_maps_and_convs(layout, grid, occupancy):
    """One cell of the occupancy x width sweep, batch 16, every width (up to 10M rows x 1024
    channels). The kernel map is compared bit-exactly with the oracle's. Each conv is compared
    with the fp32 oracle on 1024 sampled rows and, for every row, through random projections of
    the output channels (tests/fullsize.py), both as max relative error <= 1e-2."""

    dtype = torch.bfloat16
    coords = config5_coords(layout, grid, occupancy)
    c = torch.from_numpy(coords).to(DEV)
    nbr_gpu = build_neighbor_map(c, 3)
    nbr = O.build_neighbor_map(coords, 3)
    assert np.array_equal(nbr_gpu.cpu().numpy(), nbr)
    del nbr
    n = len(coords)
    rng = np.random.default_rng(grid + int(occupancy * 1000) + (7 if layout == "shell" else 0))
    rows = rng.choice(n, min(SAMPLED_ROWS, n), replace=False)
    for ch in CONFIG5_WIDTHS:
        f = device_features(n, ch, seed=ch, dtype=dtype, device=DEV)
        w = _rounded(scenes.conv_weight(ch, ch, 3, ch + 1), dtype)
        b = np.zeros(ch, np.float32)
        x = SparseTensor(f, c)
        x.cache["neighbors_3_1_(1, 1, 1)"] = nbr_gpu
        out = _conv(ch, ch, w, b, dtype)(x).features
        N.check_device_status(DEV)
        wk = O.spconv_weight_to_kio(w)
        ref = oracle_rows(f, nbr_gpu, rows, wk, b)
        got = out[torch.from_numpy(rows).to(DEV)].float().cpu().numpy()
        assert max_rel_err(got, ref) <= 1e-2, (ch, "sampled rows")
        err = projection_error(out, f, nbr_gpu, torch.from_numpy(wk), None)
        assert err <= 1e-2, (ch, "all rows", err)
        del f, x, out
    torch.cuda.empty_cache()
