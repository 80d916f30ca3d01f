"""Topology producers on the GPU: sparse_subdivide, attention windows (+ the attention calls that
use them) and occupancy -> coordinates, against the fixtures made by the reference's own code and
against the oracle at full size. Integer outputs are compared bit-exactly."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mlx_diffuser_b200 import _native as N
from mlx_diffuser_b200 import scenes
from mlx_diffuser_b200.layers.sparse import (
    SparseTensor,
    _attention_groups,
    attention_windows,
    occupied_coordinates,
    sparse_cross_attention,
    sparse_self_attention,
    sparse_subdivide,
)
from oracle import sparse_oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _t(a, dtype=None):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


# ---- sparse_subdivide -----------------------------------------------------------------------


def test_subdivide_matches_reference(topology_golden):
    g = topology_golden
    x = SparseTensor(_t(g["sub_features_in"]), _t(g["sub_coords_in"]), spatial_shape=(11, 12, 13),
                     scale=(4, 1, 2))
    x.cache["neighbors_3_1_(4, 1, 2)"] = "parent map"
    y = sparse_subdivide(x)
    assert np.array_equal(y.coords.cpu().numpy(), g["sub_coords"])
    assert np.array_equal(y.features.cpu().numpy(), g["sub_features"])
    assert y.spatial_shape == tuple(int(v) for v in g["sub_spatial_shape"])
    assert y.scale == tuple(int(v) for v in g["sub_scale"])
    assert y.cache == {} and y.batch_size == x.batch_size
    N.check_device_status(DEV)


@pytest.mark.parametrize("channels,dtype", [(64, torch.bfloat16), (3, torch.float32),
                                            (0, torch.float32)])
def test_subdivide_full_size(channels, dtype):
    coords = scenes.scene128(2)
    feats = scenes.normal_features(len(coords), channels, seed=5)
    x = SparseTensor(_t(feats, dtype), _t(coords))
    y = sparse_subdivide(x)
    want_c, want_f = O.subdivide(coords, x.features.float().cpu().numpy())
    assert np.array_equal(y.coords.cpu().numpy(), want_c)
    assert np.array_equal(y.features.float().cpu().numpy(), want_f)
    assert y.features.dtype == dtype


def test_subdivide_empty_and_wrapping():
    e = sparse_subdivide(SparseTensor(torch.zeros((0, 5), device=DEV),
                                      torch.zeros((0, 4), dtype=torch.int32, device=DEV)))
    assert tuple(e.coords.shape) == (0, 4) and tuple(e.features.shape) == (0, 5)
    big = np.array([[0, 2**30 + 3, -(2**30) - 1, 7]], np.int32)  # 2*c wraps in int32
    y = sparse_subdivide(SparseTensor(torch.ones((1, 2), device=DEV), _t(big)))
    want, _ = O.subdivide(big, np.ones((1, 2), np.float32))
    assert np.array_equal(y.coords.cpu().numpy(), want)


# ---- attention windows ----------------------------------------------------------------------


def _window_cases(g):
    i = 0
    while f"win{i}_perm" in g:
        w = int(g[f"win{i}_window"])
        yield i, (None if w < 0 else w), tuple(int(v) for v in g[f"win{i}_shift"])
        i += 1


def test_attention_groups_match_reference(topology_golden):
    g = topology_golden
    x = SparseTensor(torch.zeros((len(g["win_coords"]), 1), device=DEV), _t(g["win_coords"]))
    for i, window, shift in _window_cases(g):
        groups = attention_windows(x, window, shift)
        assert np.array_equal(groups.perm.cpu().numpy(), g[f"win{i}_perm"])
        assert np.array_equal(groups.offsets.cpu().numpy(), g[f"win{i}_offsets"])
        assert f"attention_groups_{window}_{shift}_{x.scale}" in x.cache
        listed = _attention_groups(x, window, shift)
        assert len(listed) == len(g[f"win{i}_offsets"]) - 1
    N.check_device_status(DEV)


@pytest.mark.parametrize("window,shift", [(8, (0, 0, 0)), (8, (4, 4, 4)), (5, (-3, 2, 11)),
                                          (None, (0, 0, 0))])
def test_attention_groups_full_size(window, shift):
    coords = scenes.batched([scenes.scene128(3), scenes.shell64(4), scenes.uniform(64, 0.02, 5)])
    coords = coords - np.array([0, 40, 3, 70], np.int32)  # negative coordinates
    x = SparseTensor(torch.zeros((len(coords), 1), device=DEV), _t(coords))
    got = attention_windows(x, window, shift)
    want = O.attention_groups(coords, window, shift)
    assert got.num_groups == len(want)
    assert np.array_equal(got.perm.cpu().numpy(), np.concatenate(want))
    offsets = np.cumsum([0] + [len(w) for w in want])
    assert np.array_equal(got.offsets.cpu().numpy(), offsets)


def test_attention_groups_edge_cases():
    empty = SparseTensor(torch.zeros((0, 1), device=DEV),
                         torch.zeros((0, 4), dtype=torch.int32, device=DEV))
    g = attention_windows(empty, 8)
    assert g.num_groups == 0 and g.perm.numel() == 0
    one = SparseTensor(torch.zeros((1, 1), device=DEV), _t(np.array([[3, -1, -1, -1]], np.int32)))
    g = attention_windows(one, 2, (1, 1, 1))
    assert g.num_groups == 1 and g.perm.tolist() == [0]
    with pytest.raises(ValueError, match="window_size"):
        attention_windows(one, 0)


def test_self_and_cross_attention_match_reference(topology_golden):
    g = topology_golden
    x = SparseTensor(torch.zeros((len(g["win_coords"]), 1), device=DEV), _t(g["win_coords"]))
    q, k, v = (_t(g[name]) for name in ("attn_q", "attn_k", "attn_v"))
    cases = list(_window_cases(g))[1:3]
    for j, (_, window, shift) in enumerate(cases):
        out = sparse_self_attention(x, q, k, v, window_size=window, shift_window=shift)
        np.testing.assert_allclose(out.cpu().numpy(), g[f"attn{j}_out"], rtol=1e-4, atol=1e-5)
    xb = SparseTensor(torch.zeros((len(g["cross_coords"]), 1), device=DEV), _t(g["cross_coords"]))
    out = sparse_cross_attention(xb, q, _t(g["cross_k"]), _t(g["cross_v"]))
    np.testing.assert_allclose(out.cpu().numpy(), g["cross_out"], rtol=1e-4, atol=1e-5)
    with pytest.raises(ValueError, match="share shape"):
        sparse_self_attention(x, q, k[:-1], v)


# ---- occupancy -> coordinates ---------------------------------------------------------------


def test_occupied_coordinates_match_reference(topology_golden):
    g = topology_golden
    logits = _t(g["occ_logits"])
    for i in range(3):
        got = occupied_coordinates(logits, float(g[f"occ{i}_threshold"]))
        assert np.array_equal(got.cpu().numpy(), g[f"occ{i}_coords"])
    half = _t(g["occ_half_logits"])  # float16
    got = occupied_coordinates(half, float(g["occ_half_threshold"]))
    assert np.array_equal(got.cpu().numpy(), g["occ_half_coords"])
    N.check_device_status(DEV)


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_occupied_coordinates_full_size(dtype):
    rng = np.random.default_rng(8)
    logits = rng.standard_normal((16, 64, 64, 64)).astype(np.float32) - 1.6  # ~5.5% occupied
    tdtype = getattr(torch, dtype)
    t = torch.from_numpy(logits).to(DEV, tdtype)
    exact = t.float().cpu().numpy()  # the values the kernel compares
    for thr in (0.0, 0.3):
        got = occupied_coordinates(t, thr)
        want = O.occupied_coordinates(exact, thr, dtype)
        assert np.array_equal(got.cpu().numpy(), want)


def test_occupied_coordinates_views_and_edges():
    rng = np.random.default_rng(9)
    # channels-last decoder output: channel 0 of a (B, D, H, W, 3) tensor, read in place
    full = rng.standard_normal((2, 13, 7, 11, 3)).astype(np.float32)
    got = occupied_coordinates(_t(full), 0.25)
    assert np.array_equal(got.cpu().numpy(), O.occupied_coordinates(full[..., 0], 0.25))
    # a permuted (non-contiguous) grid
    grid = _t(rng.standard_normal((3, 9, 10, 11)).astype(np.float32))
    perm = grid.permute(0, 3, 1, 2)
    got = occupied_coordinates(perm, 0.0)
    want = O.occupied_coordinates(perm.cpu().numpy(), 0.0)
    assert np.array_equal(got.cpu().numpy(), want)
    # NaN never counts; all below; all above; empty grid
    nan = torch.full((1, 4, 4, 4), float("nan"), device=DEV)
    assert occupied_coordinates(nan, -1e30).shape == (0, 4)
    assert occupied_coordinates(torch.zeros((2, 3, 3, 3), device=DEV), 0.0).shape == (0, 4)
    ones = occupied_coordinates(torch.ones((2, 3, 4, 5), device=DEV), 0.0)
    assert np.array_equal(ones.cpu().numpy(), np.argwhere(np.ones((2, 3, 4, 5)) > 0))
    assert occupied_coordinates(torch.zeros((0, 4, 4, 4), device=DEV)).shape == (0, 4)
    with pytest.raises(ValueError, match="occupancy logits"):
        occupied_coordinates(torch.zeros((4, 4, 4), device=DEV))
    N.check_device_status(DEV)
