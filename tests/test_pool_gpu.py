"""Sparse downsample / upsample on the GPU against the reference (bit-exact integers)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mlx_diffuser_b200 import _native as N
from mlx_diffuser_b200 import scenes
from mlx_diffuser_b200.layers.sparse import SparseTensor, sparse_downsample, sparse_upsample
from oracle import sparse_oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _tensor(coords, feats, dtype=torch.float32, spatial_shape=None):
    return SparseTensor(
        torch.from_numpy(np.ascontiguousarray(feats)).to(DEV, dtype),
        torch.from_numpy(np.ascontiguousarray(coords)).to(DEV),
        spatial_shape=spatial_shape,
    )


def test_down_up_match_golden(golden):
    _, g = golden
    factors = sorted(int(k[4:-7]) for k in g if k.startswith("down") and k.endswith("_coords"))
    for f in factors:
        x = _tensor(g["coords"], g["features"],
                    spatial_shape=tuple(int(v) for v in g["spatial_shape"]))
        down = sparse_downsample(x, f)
        up = sparse_upsample(down, f)
        assert np.array_equal(down.coords.cpu().numpy(), g[f"down{f}_coords"])
        inverse = down.cache[f"upsample_{f}_{down.scale}"][1]
        assert np.array_equal(inverse.cpu().numpy(), g[f"down{f}_inverse"])
        # fp32 sums run in fine-row order, like the reference's scatter-add: bit-exact
        assert np.array_equal(down.features.cpu().numpy(), g[f"down{f}_features"])
        assert np.array_equal(up.features.cpu().numpy(), g[f"up{f}_features"])
        assert down.spatial_shape == tuple(int(v) for v in g[f"down{f}_spatial_shape"])
        assert down.scale == tuple(int(v) for v in g[f"down{f}_scale"])
        assert torch.equal(up.coords, x.coords) and up.scale == x.scale
    N.check_device_status(DEV)


def test_reference_block_test():
    """``tests/test_trellis.py:147-161``: a 2^3 block pools to one voxel holding sum / 9."""

    coords = np.array([[0, z, y, x] for z in range(2) for y in range(2) for x in range(2)], np.int32)
    feats = np.arange(16, dtype=np.float32).reshape(8, 2)
    x = _tensor(coords, feats, spatial_shape=(2, 2, 2))
    down = sparse_downsample(x)
    up = sparse_upsample(down)
    assert tuple(down.coords.shape) == (1, 4)
    assert tuple(up.coords.shape) == tuple(x.coords.shape)
    pooled = feats.sum(0) / 9
    np.testing.assert_allclose(up.features.cpu().numpy(), np.broadcast_to(pooled, (8, 2)), rtol=1e-6)


@pytest.mark.parametrize("name", ["shell64", "scene128", "uniform128_8pct_b4", "negative_f3"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_full_size_matches_oracle(name, dtype):
    factor = 3 if name == "negative_f3" else 2
    coords = {
        "shell64": lambda: scenes.shell64(1),
        "scene128": lambda: scenes.scene128(1),
        "uniform128_8pct_b4": lambda: scenes.batched(
            [scenes.uniform(128, 0.08, 40 + b) for b in range(4)]
        ),
        "negative_f3": lambda: scenes.shell64(2) - np.array([0, 40, 31, 7], np.int32),
    }[name]()
    feats = scenes.normal_features(len(coords), 24, seed=7)
    x = _tensor(coords, feats, dtype)
    down = sparse_downsample(x, factor)
    want_c, want_inv = O.downsample_coords(coords, factor)
    assert np.array_equal(down.coords.cpu().numpy(), want_c)
    inv = down.cache[f"upsample_{factor}_{down.scale}"][1].cpu().numpy()
    assert np.array_equal(inv, want_inv)
    f_in = x.features.float().cpu().numpy()
    ref = O.downsample_features(f_in, want_inv, len(want_c))
    got = down.features.float().cpu().numpy()
    if dtype == torch.float32:
        assert np.array_equal(got, ref)
    else:
        assert np.abs(got - ref).max() / np.abs(ref).max() <= 1e-2
    up = sparse_upsample(down, factor)
    assert torch.equal(up.features, down.features[torch.from_numpy(inv).long().to(DEV)])


def test_pool_edge_cases():
    empty = _tensor(np.zeros((0, 4), np.int32), np.zeros((0, 3), np.float32))
    down = sparse_downsample(empty)
    assert tuple(down.coords.shape) == (0, 4) and tuple(down.features.shape) == (0, 3)
    assert sparse_upsample(down).features.shape == (0, 3)
    # multi-dimensional features and an odd channel count (scalar path)
    coords = scenes.shell(16, 5.5, 2.0, 1.0, seed=1)
    feats = scenes.normal_features(len(coords), 15, seed=2).reshape(len(coords), 3, 5)
    x = SparseTensor(torch.from_numpy(feats).to(DEV), torch.from_numpy(coords).to(DEV))
    down = sparse_downsample(x)
    c, inv = O.downsample_coords(coords, 2)
    ref = O.downsample_features(feats.reshape(len(coords), 15), inv, len(c)).reshape(len(c), 3, 5)
    assert np.array_equal(down.features.cpu().numpy(), ref)
    assert sparse_upsample(down).features.shape == x.features.shape
    # factor 1 keeps unique rows, sorted
    d1 = sparse_downsample(x, 1)
    assert np.array_equal(d1.coords.cpu().numpy(), O.downsample_coords(coords, 1)[0])
    with pytest.raises(ValueError, match="positive"):
        sparse_downsample(x, 0)
    N.check_device_status(DEV)
