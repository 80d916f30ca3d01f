"""Kernel map on the GPU: bit-exact against the reference's build_neighbor_map.

Golden fixtures come from the reference's own code; full-size scenes are checked against the
oracle (itself pinned to the fixtures in test_oracle.py).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mlx_diffuser_b200 import _native as N
from mlx_diffuser_b200 import scenes
from mlx_diffuser_b200.layers.sparse import build_neighbor_map, conv_row_order
from oracle import sparse_oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _gpu_map(coords, ks=3, dl=1, **kw):
    out = build_neighbor_map(torch.from_numpy(np.ascontiguousarray(coords)).to(DEV), ks, dl, **kw)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_kmap_matches_golden(golden):
    _, g = golden
    assert np.array_equal(_gpu_map(g["coords"], int(g["kernel_size"]), int(g["dilation"])), g["nbr"])
    i = 0
    while f"nbr_extra{i}" in g:
        ks = tuple(int(v) for v in g[f"nbr_extra{i}_kernel"])
        dl = tuple(int(v) for v in g[f"nbr_extra{i}_dilation"])
        assert np.array_equal(_gpu_map(g["coords"], ks, dl), g[f"nbr_extra{i}"])
        i += 1


@pytest.mark.parametrize(
    "name",
    ["shell64", "shell32x4", "scene128", "uniform64_30pct", "uniform128_2pct_b16"],
)
def test_kmap_full_size_matches_oracle(name):
    coords = {
        "shell64": lambda: scenes.shell64(0),
        "shell32x4": lambda: scenes.shell32_batch(4),
        "scene128": lambda: scenes.scene128(0),
        "uniform64_30pct": lambda: scenes.uniform(64, 0.30, 5),
        "uniform128_2pct_b16": lambda: scenes.batched(
            [scenes.uniform(128, 0.02, 100 + b) for b in range(16)]
        ),
    }[name]()
    want = O.build_neighbor_map(coords, 3)
    got = _gpu_map(coords)
    assert np.array_equal(got, want)


def test_kmap_edge_cases_match_dict_oracle():
    imax, imin = np.iinfo(np.int32).max, np.iinfo(np.int32).min
    c = np.array(
        [
            [0, imax, 0, 0],
            [0, imax - 1, 0, 0],
            [0, imin, imin, imin],
            [0, imin + 1, imin, imin],
            [-3, 5, 5, 5],     # negative batch index is just another key
            [-3, 5, 6, 5],
            [7, 0, 0, 0],
            [7, 0, 0, 0],      # duplicate rows: the later row wins
            [7, 0, 0, 1],
            [7, 0, 0, 0],
        ],
        np.int32,
    )
    for ks, dl in ((3, 1), ((3, 1, 5), (2, 1, 1)), (1, 1), (5, 3)):
        want = O.build_neighbor_map_dict(c, ks, dl)
        assert np.array_equal(_gpu_map(c, ks, dl), want), (ks, dl)
    m = _gpu_map(c)
    assert m[7, 13] == 9 and m[9, 13] == 9


def test_block_table_edge_values_match_dict_oracle():
    """The 3x3x3 map goes through the 2x2x2-block table: blocks straddling zero (negative
    coordinates floor-divide), every corner of the int32 range, batch index -1 (the empty slot's
    pattern) and 0x7F7F7F7F, duplicates spread over several blocks, and a dense random cloud with
    many duplicates -- all against the reference's dict restated on the CPU."""

    imax, imin = np.iinfo(np.int32).max, np.iinfo(np.int32).min
    rows = []
    for marker in (-1, 0x7F7F7F7F):
        rows += [[marker, 0, 0, 0], [marker, 1, 1, 1], [marker, 0, 0, 0], [marker, -1, 0, 0],
                 [marker, -1, -1, -1], [marker, -2, -2, -2]]
    for cx in (imin, imin + 1, imax - 1, imax):
        for cy in (imin, imax):
            for cz in (imin + 1, imax - 1):
                rows.append([2, cx, cy, cz])
    edge = np.array(rows, np.int32)
    assert np.array_equal(_gpu_map(edge), O.build_neighbor_map_dict(edge, 3))
    rng = np.random.default_rng(21)
    cloud = rng.integers(-4, 4, size=(3000, 4)).astype(np.int32)
    cloud[:, 0] = rng.integers(-2, 2, size=3000)
    want = O.build_neighbor_map_dict(cloud, 3)
    assert np.array_equal(_gpu_map(cloud), want)


def test_kmap_empty_and_single():
    assert _gpu_map(np.zeros((0, 4), np.int32)).shape == (0, 27)
    single = _gpu_map(np.array([[0, 3, 4, 5]], np.int32))
    assert single[0, 13] == 0 and (np.delete(single[0], 13) == -1).all()


def test_kmap_undersized_table_raises():
    coords = scenes.shell(16, 5.5, 2.0, 1.0, seed=3)
    assert len(coords) > 64
    with pytest.raises(RuntimeError, match="hash table full"):
        _gpu_map(coords, table_slots=64)
    # a correctly sized explicit table works and leaves the status clean
    assert np.array_equal(_gpu_map(coords, table_slots=4096), O.build_neighbor_map(coords, 3))


def test_conv_row_order_groups_rows_by_mask():
    coords = scenes.shell32_batch(2)
    nbr = build_neighbor_map(torch.from_numpy(coords).to(DEV), 3)
    order_t, tiles_t = conv_row_order(nbr)
    order = order_t.cpu().numpy()
    n = len(coords)
    assert np.array_equal(np.sort(order), np.arange(n))
    host = nbr.cpu().numpy()
    masks = ((host >= 0).astype(np.int64) << np.arange(27)).sum(1)
    m = masks[order]
    assert (np.diff(m) >= 0).all()
    same = np.diff(m) == 0
    assert (np.diff(order)[same] > 0).all()  # stable: spatial order kept inside a group
    # tiles listed most expensive first: non-increasing union popcount, a permutation
    tiles = tiles_t.cpu().numpy()
    assert np.array_equal(np.sort(tiles), np.arange(-(-n // 128)))
    cost = [bin(int(np.bitwise_or.reduce(m[t * 128:(t + 1) * 128]))).count("1") for t in tiles]
    assert all(a >= b for a, b in zip(cost, cost[1:]))
    assert conv_row_order(build_neighbor_map(torch.from_numpy(coords).to(DEV), 5)) == (None, None)
    N.check_device_status(DEV)


def _expected_schedule(nbr: np.ndarray):
    """A stable sort of the row masks, then a stable sort of the 128-row tiles by
    32 - popcount(union of their masks)."""
    kvol = nbr.shape[1]
    masks = ((nbr >= 0).astype(np.int64) << np.arange(kvol)).sum(1)
    order = np.argsort(masks, kind="stable")
    m = masks[order]
    tiles = -(-len(nbr) // 128)
    keys = np.array([32 - bin(int(np.bitwise_or.reduce(m[t * 128:(t + 1) * 128]))).count("1")
                     for t in range(tiles)])
    return order, np.argsort(keys, kind="stable")


# Row counts either side of the one-cluster schedule's run lengths (2048 and 4096 rows), its
# switch to 16-CTA clusters (16384) and its row limit (32768, above which the device-wide sort
# runs), with kernel volumes 27, 9 and 32.
@pytest.mark.parametrize("n,kvol", [(1, 27), (127, 27), (2048, 27), (2049, 27), (4097, 27),
                                    (16384, 27), (16385, 27), (24168, 27), (32768, 27),
                                    (32769, 27), (70001, 27), (20000, 9), (30000, 32)])
def test_conv_row_order_is_the_stable_sort(n, kvol):
    rng = np.random.default_rng(n + kvol)
    # few distinct masks (long runs of equal keys across the cluster's runs), the all-ones mask
    # (equal to the padding key of a partial run) and random masks
    pool = rng.integers(0, 2, size=(40, kvol)).astype(bool)
    pool[0] = True
    pool[1] = False
    pick = rng.integers(0, len(pool), size=n)
    present = pool[pick]
    rand = rng.random(n) < 0.2
    present[rand] = rng.random((int(rand.sum()), kvol)) < 0.7
    nbr = np.where(present, rng.integers(0, max(n, 1), size=(n, kvol)), -1).astype(np.int32)
    order_t, tiles_t = conv_row_order(torch.from_numpy(nbr).to(DEV))
    order, tiles = _expected_schedule(nbr)
    assert np.array_equal(order_t.cpu().numpy(), order)
    assert np.array_equal(tiles_t.cpu().numpy(), tiles)


# ---- dense-grid kernel map ----------------------------------------------------------------------


def test_grid_map_matches_hash_map_on_every_fixture(golden):
    """The grid path (forced) gives the hash path's map bit for bit: duplicates, negative
    coordinates, three batch elements, anisotropic kernels and dilations."""

    _, g = golden
    coords = torch.from_numpy(g["coords"]).to(DEV)
    maps = [(int(g["kernel_size"]), int(g["dilation"]), g["nbr"])]
    i = 0
    while f"nbr_extra{i}" in g:
        maps.append((tuple(int(v) for v in g[f"nbr_extra{i}_kernel"]),
                     tuple(int(v) for v in g[f"nbr_extra{i}_dilation"]), g[f"nbr_extra{i}"]))
        i += 1
    for ks, dl, want in maps:
        got = build_neighbor_map(coords, ks, dl, method="grid")
        assert np.array_equal(got.cpu().numpy(), want)
        assert torch.equal(got, build_neighbor_map(coords, ks, dl, method="hash"))
    N.check_device_status(DEV)


def test_grid_map_auto_selection_on_dense_and_sparse_boxes():
    dense = scenes.batched([scenes.uniform(64, 0.08, 700 + b) for b in range(4)])  # ~84k rows
    c = torch.from_numpy(dense).to(DEV)
    assert torch.equal(build_neighbor_map(c, 3, method="grid"),
                       build_neighbor_map(c, 3, method="hash"))
    assert torch.equal(build_neighbor_map(c, 3), build_neighbor_map(c, 3, method="hash"))
    assert np.array_equal(build_neighbor_map(c, 3).cpu().numpy(), O.build_neighbor_map(dense, 3))
    # far-apart batch indices make the box huge: auto keeps the hash table
    sparse = dense.copy()
    sparse[:, 0] *= 100000
    c2 = torch.from_numpy(sparse).to(DEV)
    assert np.array_equal(build_neighbor_map(c2, 3).cpu().numpy(), O.build_neighbor_map(sparse, 3))
    N.check_device_status(DEV)


def _box_rows(shape, n_unique: int, dup: int) -> np.ndarray:
    """`n_unique` distinct rows in a box of `shape` (batch, c1, c2, c3), both corners occupied,
    plus `dup` repeated rows, shuffled. Every spatial range starts at an even coordinate and has
    an even length, so the box is whole 2x2x2 blocks and the block grid of a 3x3x3 map has as
    many cells as the voxel grid."""
    rng = np.random.default_rng(dup + n_unique)
    cells = int(np.prod(shape))
    flat = rng.choice(cells, size=n_unique - 2, replace=False)
    b, rest = np.divmod(flat, shape[1] * shape[2] * shape[3])
    c1, rest = np.divmod(rest, shape[2] * shape[3])
    c2, c3 = np.divmod(rest, shape[3])
    lo = np.array([0, -8, 100, -50])
    rows = np.stack([b, c1, c2, c3], 1) + lo
    corners = np.array([lo, lo + np.array(shape) - 1])
    rows = np.concatenate([rows, corners]).astype(np.int32)
    rows = np.concatenate([rows, rows[rng.choice(n_unique, dup)]])
    return rows[rng.permutation(len(rows))]


# From 2^17 rows the device picks the grid at <= 16 cells per row and the hash table above: a
# 4 x 64 x 64 x 144 box (2,359,296 cells) with 147,456 rows is exactly 16 cells per row, one row
# fewer is just above; for the 3x3x3 block path and the general (kernel, dilation) path.
@pytest.mark.parametrize("dup", [64, 63])
@pytest.mark.parametrize("ks,dl", [(3, 1), (3, 2), ((3, 1, 5), (1, 2, 1))])
def test_auto_map_either_side_of_the_grid_limit(dup, ks, dl):
    rows = _box_rows((4, 64, 64, 144), 147456 - 64, dup)
    assert len(rows) >= 1 << 17
    got = _gpu_map(rows, ks, dl)
    assert np.array_equal(got, O.build_neighbor_map(rows, ks, dl))
    c = torch.from_numpy(rows).to(DEV)
    assert np.array_equal(got, build_neighbor_map(c, ks, dl, method="hash").cpu().numpy())
    N.check_device_status(DEV)


# Below 2^17 rows the automatic map always takes the hash table.
@pytest.mark.parametrize("ks,dl", [(3, 1), (5, 1), ((3, 1, 5), (1, 2, 1))])
def test_auto_map_small_box(ks, dl):
    rows = _box_rows((2, 16, 16, 18), 512, 64)
    assert np.array_equal(_gpu_map(rows, ks, dl), O.build_neighbor_map_dict(rows, ks, dl))
    N.check_device_status(DEV)


def test_grid_map_refuses_rows_outside_the_given_box():
    import ctypes

    coords = torch.tensor([[0, 0, 0, 0], [0, 5, 5, 5], [0, 9, 9, 9]], dtype=torch.int32, device=DEV)
    lib = N.load()
    ext = (ctypes.c_int64 * 4)(1, 6, 6, 6)  # too small for the last row
    ws = torch.empty(lib.sv_kmap_grid_workspace_bytes(ext), dtype=torch.uint8, device=DEV)
    nbr = torch.empty((3, 27), dtype=torch.int32, device=DEV)
    int3 = ctypes.c_int * 3
    rc = lib.sv_kmap_build_grid(coords.data_ptr(), 3, int3(3, 3, 3), int3(1, 1, 1), nbr.data_ptr(),
                                (ctypes.c_int32 * 4)(0, 0, 0, 0), ext, ws.data_ptr(), ws.numel(),
                                N.status_word(DEV).data_ptr(), N.stream(DEV))
    assert rc == N.SV_OK
    with pytest.raises(RuntimeError, match="out of range"):
        N.check_device_status(DEV)
    assert int(nbr[0, 13]) == 0 and int(nbr[1, 13]) == 1 and int(nbr[2, 13]) == -1
