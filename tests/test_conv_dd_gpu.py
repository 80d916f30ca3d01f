"""The deduplicated-tile convolution for narrow channels (``sv_conv_dd_plan`` +
``sv_conv3d_forward_dd``) against the fp32 oracle of the reference's convolution
(``src/mlx_diffuser/kernels/sparse.py:39-55``), and its tile plan against a NumPy restatement.

The plan is integer data and is compared exactly: tiles of 128 rows in (batch, Morton) order,
each tile's distinct source rows in that order too, every local-map entry pointing at its source
row (or -1 / -2 for a missing neighbour / a row the 56 KB buffer could not hold)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mlx_diffuser_b200 import _native as N
from mlx_diffuser_b200 import scenes
from mlx_diffuser_b200.kernels.sparse import DedupPlan, conv3d_forward_dd
from mlx_diffuser_b200.layers.sparse import SparseConv3D, SparseTensor, build_neighbor_map
from oracle import sparse_oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
HALF_TOL = 1e-2


def max_rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def _rounded(a, dtype):
    return torch.from_numpy(np.asarray(a, np.float32)).to(dtype).float().numpy()


def _spread3(v: np.ndarray) -> np.ndarray:
    v = v.astype(np.uint64) & np.uint64(0xFFFF)
    out = np.zeros_like(v)
    for i in range(16):
        out |= ((v >> np.uint64(i)) & np.uint64(1)) << np.uint64(3 * i)
    return out


def morton_rows(coords: np.ndarray) -> np.ndarray:
    """Row order of the plan: stable sort by batch (15 bits) over the Morton code of the low 16
    bits of the three spatial columns (first spatial column most significant)."""

    c = coords.astype(np.int64)
    key = ((c[:, 0].astype(np.uint64) & np.uint64(0x7FFF)) << np.uint64(48)) | (
        _spread3(c[:, 1]) << np.uint64(2)) | (_spread3(c[:, 2]) << np.uint64(1)) | _spread3(c[:, 3])
    return np.argsort(key, kind="stable")


def decode_plan(plan: DedupPlan):
    lib = N.load()
    n, cin = plan.n, plan.cin
    tiles = (n + 127) // 128
    umax = 56 * 1024 // (2 * cin)  # rows one shared-memory buffer of the kernel holds
    raw = plan.buffer.cpu().numpy()
    align = lambda v: (v + 255) // 256 * 256  # noqa: E731
    o = 0
    rows = raw[o : o + tiles * 128 * 4].view(np.int32).reshape(tiles, 128)
    o += align(tiles * 128 * 4)
    lnbr = raw[o : o + tiles * 128 * 27 * 2].view(np.int16).reshape(tiles, 128, 27)
    o += align(tiles * 128 * 27 * 2)
    src = raw[o : o + tiles * umax * 4].view(np.int32).reshape(tiles, umax)
    o += align(tiles * umax * 4)
    meta = raw[o : o + tiles * 16].view(np.int32).reshape(tiles, 4)
    assert int(lib.sv_conv_dd_plan_bytes(n, cin)) == plan.nbytes
    return rows, lnbr, src, meta, umax


def check_plan(coords: np.ndarray, nbr: np.ndarray, plan: DedupPlan) -> int:
    """Exact check of the plan; returns the number of local-map entries that overflowed. A
    tile's distinct source rows are listed in Morton order (their rank in the row order)."""

    rows, lnbr, src, meta, umax = decode_plan(plan)
    n = len(coords)
    morton = morton_rows(coords)
    rank = np.empty(n, np.int64)
    rank[morton] = np.arange(n)
    order = np.full(rows.size, -1, np.int64)
    order[:n] = morton
    assert np.array_equal(rows.reshape(-1), order)
    overflow = 0
    for t in range(rows.shape[0]):
        r = rows[t]
        valid = r >= 0
        nb = np.full((128, 27), -1, np.int64)
        nb[valid] = nbr[r[valid]]
        ranks = np.unique(rank[nb[nb >= 0]])
        assert meta[t, 2] == len(ranks)
        assert meta[t, 0] == min(len(ranks), umax)
        assert meta[t, 1] == int(np.bitwise_or.reduce(
            ((nb >= 0) << np.arange(27)).astype(np.int64).sum(1).astype(np.int64)))
        kept = min(len(ranks), umax)
        assert np.array_equal(src[t, :kept], morton[ranks[:kept]])
        assert (src[t, kept:] == -1).all()
        slot = np.searchsorted(ranks, rank[np.maximum(nb, 0)])
        want = np.where(nb < 0, -1, np.where(slot < umax, slot, -2))
        assert np.array_equal(lnbr[t].astype(np.int64), want)
        overflow += int((want == -2).sum())
    return overflow


def _dd_conv(coords, f, w_oki, b, dtype, residual=None, plan_out=None):
    c = torch.from_numpy(coords).to(DEV)
    nbr = build_neighbor_map(c, 3)
    feats = torch.from_numpy(f).to(DEV, dtype)
    w = torch.from_numpy(w_oki).to(DEV, dtype).contiguous()
    bias = None if b is None else torch.from_numpy(b).to(DEV, dtype)
    plan = DedupPlan(c, nbr, f.shape[1])
    res = None if residual is None else torch.from_numpy(residual).to(DEV, dtype)
    out = conv3d_forward_dd(feats, nbr, plan, w, bias, w_oki.shape[0], residual=res)
    torch.cuda.synchronize()
    N.check_device_status(DEV)
    if plan_out is not None:
        plan_out.append(plan)
    return out.float().cpu().numpy(), nbr.cpu().numpy()


@pytest.mark.parametrize("cin,cout", [(64, 64), (64, 32), (64, 128), (64, 96), (128, 128),
                                      (128, 64), (128, 32), (128, 256)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_dd_conv_matches_oracle(cin, cout, dtype):
    coords = scenes.batched([scenes.shell(20, 7.0, 2.5, 1.0, seed=3),
                             scenes.shell(16, 5.5, 2.0, 1.0, seed=4)])
    f = _rounded(scenes.normal_features(len(coords), cin, seed=5), dtype)
    w = _rounded(scenes.conv_weight(cout, cin, 3, seed=6), dtype)
    b = _rounded(np.random.default_rng(7).standard_normal(cout) * 0.1, dtype)
    plans = []
    out, nbr = _dd_conv(coords, f, w, b, dtype, plan_out=plans)
    assert np.array_equal(nbr, O.build_neighbor_map(coords, 3))
    ref = O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w), b)
    assert max_rel_err(out, ref) <= HALF_TOL
    check_plan(coords, nbr, plans[0])


def test_dd_plan_and_conv_on_scene128():
    """The config-4 scene (~237k rows, 1849 tiles): plan exact, 64 -> 64 conv within 1e-2."""

    dtype = torch.bfloat16
    coords = scenes.scene128(0)
    f = _rounded(scenes.normal_features(len(coords), 64, seed=40), dtype)
    w = _rounded(scenes.conv_weight(64, 64, 3, 41), dtype)
    plans = []
    out, nbr = _dd_conv(coords, f, w, None, dtype, plan_out=plans)
    ref = O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w), np.zeros(64, np.float32))
    assert max_rel_err(out, ref) <= HALF_TOL
    check_plan(coords, nbr, plans[0])


def test_dd_overflow_rows_are_read_from_global_memory():
    """A dense 24^3 box at 128 channels: a 128-row Morton tile (4 x 4 x 8 cells) references
    6 x 6 x 10 = 360 distinct rows, more than the 256 the buffer holds at 256 bytes per row; the
    rest are read from global memory through the map. The result must not change."""

    dtype = torch.bfloat16
    g = np.stack(np.meshgrid(np.arange(24), np.arange(24), np.arange(24), indexing="ij"), -1)
    coords = np.zeros((24**3, 4), np.int32)
    coords[:, 1:] = g.reshape(-1, 3)
    coords = coords[np.random.default_rng(1).permutation(len(coords))]
    f = _rounded(scenes.normal_features(len(coords), 128, seed=2), dtype)
    w = _rounded(scenes.conv_weight(64, 128, 3, 3), dtype)
    plans = []
    out, nbr = _dd_conv(coords, f, w, None, dtype, plan_out=plans)
    overflow = check_plan(coords, nbr, plans[0])
    assert overflow > 0
    ref = O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w), np.zeros(64, np.float32))
    assert max_rel_err(out, ref) <= HALF_TOL


def test_dd_residual_and_edge_sizes():
    dtype = torch.bfloat16
    for n_rows in (1, 127, 128, 129, 257):
        coords = scenes.shell(16, 5.5, 2.0, 1.0, seed=11)[:n_rows]
        f = _rounded(scenes.normal_features(len(coords), 64, seed=12), dtype)
        w = _rounded(scenes.conv_weight(64, 64, 3, 13), dtype)
        b = _rounded(np.linspace(-1, 1, 64), dtype)
        res = _rounded(scenes.normal_features(len(coords), 64, seed=14), dtype)
        out, nbr = _dd_conv(coords, f, w, b, dtype, residual=res)
        ref = O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w), b) + res
        assert max_rel_err(out, ref) <= HALF_TOL, n_rows
    # isolated points: only the centre offset is valid
    coords = np.zeros((300, 4), np.int32)
    coords[:, 1] = np.arange(300) * 3
    f = _rounded(scenes.normal_features(300, 64, seed=15), dtype)
    w = _rounded(scenes.conv_weight(32, 64, 3, 16), dtype)
    out, nbr = _dd_conv(coords, f, w, None, dtype)
    ref = O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w), np.zeros(32, np.float32))
    assert max_rel_err(out, ref) <= HALF_TOL


def test_module_auto_picks_dedup_for_surfaces_and_matches_mask_sorted_kernel():
    """SparseConv3D under AUTO runs the deduplicated kernel on a surface (many neighbours per
    row) and caches its plan; forcing the mask-sorted tcgen05 kernel gives the same output
    (both accumulate each row's terms offset by offset in fp32; agreement to 1e-6)."""

    dtype = torch.bfloat16
    coords = scenes.shell32_batch(4)
    x = SparseTensor(torch.from_numpy(scenes.normal_features(len(coords), 64, 1)).to(DEV, dtype),
                     torch.from_numpy(coords).to(DEV))
    conv = SparseConv3D(64, 64).to(DEV)
    conv.conv.weight = torch.from_numpy(scenes.conv_weight(64, 64, 3, 2)).to(DEV, dtype)
    conv.conv.bias = torch.zeros(64, device=DEV, dtype=dtype)
    auto = conv(x).features
    assert any(str(k).startswith("conv_dd64") for k in x.cache)
    conv.algo = N.SV_CONV_TCGEN05
    plain = conv(x).features
    N.check_device_status(DEV)
    assert max_rel_err(auto.float().cpu(), plain.float().cpu()) <= 1e-6
