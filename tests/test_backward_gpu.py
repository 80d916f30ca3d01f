"""Backward pass of the submanifold convolution on the GPU against the gradient oracle (which
is pinned to torch autograd of the reference's fallback formula): pair lists, the flipped
weight, input / weight / bias gradients on both kernel paths, and autograd through
SparseConv3D."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mlx_diffuser_b200 import _native as N
from mlx_diffuser_b200 import scenes
from mlx_diffuser_b200.kernels.sparse import (
    conv3d_dbias,
    conv3d_dgrad,
    conv3d_wgrad,
    kmap_pairs,
    weight_flip_transpose,
)
from mlx_diffuser_b200.layers.sparse import (
    MapTopology,
    SparseConv3D,
    SparseTensor,
    build_neighbor_map,
    conv_row_order,
)
from oracle import sparse_oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
HALF_TOL = 1e-2


def _t(a, dtype=None):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def _rounded(a, dtype):
    return torch.from_numpy(np.asarray(a, np.float32)).to(dtype).float().numpy()


def max_rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def _oki_to_kio_grad(dw_oki: np.ndarray) -> np.ndarray:
    o = dw_oki.shape[0]
    i = dw_oki.shape[-1]
    return dw_oki.reshape(o, -1, i).transpose(1, 2, 0)


def _grads(features, nbr, weight_oki, dout, unique, algo=N.SV_CONV_AUTO):
    """Library gradients for spconv-layout weights; returns numpy (dx, dw_kio, db)."""

    nb = _t(nbr)
    ro, to = conv_row_order(nb)
    dx = conv3d_dgrad(dout, nb, weight_oki, unique=unique, row_order=ro, tile_order=to, algo=algo)
    dw = conv3d_wgrad(features, dout, kmap_pairs(nb), weight_oki.shape[1:4], algo=algo)
    db = conv3d_dbias(dout)
    N.check_device_status(DEV)
    return (dx.float().cpu().numpy(), _oki_to_kio_grad(dw.float().cpu().numpy()),
            db.float().cpu().numpy())


def test_pair_lists_match_the_map(golden):
    _, g = golden
    nbr = g["nbr"]
    offsets, src, dst = kmap_pairs(_t(nbr))
    off = offsets.cpu().numpy()
    src, dst = src.cpu().numpy(), dst.cpu().numpy()
    assert off[0] == 0 and off[-1] == int((nbr >= 0).sum())
    for k in range(nbr.shape[1]):
        want_dst = np.nonzero(nbr[:, k] >= 0)[0]
        assert np.array_equal(dst[off[k]:off[k + 1]], want_dst)
        assert np.array_equal(src[off[k]:off[k + 1]], nbr[want_dst, k])
    empty = kmap_pairs(torch.zeros((0, 27), dtype=torch.int32, device=DEV))
    assert empty[0].tolist() == [0] * 28 and empty[1].numel() == 0
    N.check_device_status(DEV)


def test_weight_flip_transpose():
    w = np.random.default_rng(0).standard_normal((5, 3, 1, 5, 7)).astype(np.float32)
    got = weight_flip_transpose(_t(w)).cpu().numpy()
    want = w[:, ::-1, ::-1, ::-1, :].transpose(4, 1, 2, 3, 0)
    assert np.array_equal(got, want)


def test_fp32_gradients_match_oracle(golden):
    """CUDA-core paths in fp32 on every reference fixture: duplicates (the resolved-row input
    gradient), negative coordinates, kernel 5, dilation 2."""

    _, g = golden
    rng = np.random.default_rng(11)
    f, nbr, w = g["features"], g["nbr"], g["weight"]
    dout = rng.standard_normal((len(nbr), w.shape[0])).astype(np.float32)
    unique = bool(np.all(nbr[:, nbr.shape[1] // 2] == np.arange(len(nbr))))
    dx, dw, db = _grads(_t(f), nbr, _t(w), _t(dout), unique)
    rx, rw, rb = O.sparse_conv3d_grads(f, nbr, O.spconv_weight_to_kio(w), dout, accum=np.float64)
    np.testing.assert_allclose(dx, rx, rtol=1e-4, atol=1e-4 * np.abs(rx).max())
    np.testing.assert_allclose(dw, rw, rtol=1e-4, atol=1e-4 * np.abs(rw).max())
    np.testing.assert_allclose(db, rb, rtol=1e-4, atol=1e-4 * np.abs(rb).max())
    # non-cubic kernels and dilations of the same fixture
    i = 0
    while f"nbr_extra{i}" in g:
        ks = tuple(int(v) for v in g[f"nbr_extra{i}_kernel"])
        nb2 = g[f"nbr_extra{i}"]
        w2 = rng.standard_normal((3, *ks, f.shape[1])).astype(np.float32)
        d2 = rng.standard_normal((len(nb2), 3)).astype(np.float32)
        uq = bool(np.all(nb2[:, nb2.shape[1] // 2] == np.arange(len(nb2))))
        dx, dw, _ = _grads(_t(f), nb2, _t(w2), _t(d2), uq)
        rx, rw, _ = O.sparse_conv3d_grads(f, nb2, w2.reshape(3, -1, f.shape[1]).transpose(1, 2, 0),
                                          d2, accum=np.float64)
        np.testing.assert_allclose(dx, rx, rtol=1e-4, atol=1e-4 * max(np.abs(rx).max(), 1e-6))
        np.testing.assert_allclose(dw, rw, rtol=1e-4, atol=1e-4 * max(np.abs(rw).max(), 1e-6))
        i += 1


@pytest.mark.parametrize("cin,cout", [(64, 128), (128, 256), (256, 128), (512, 512), (192, 384),
                                      (96, 128)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_gradients_tensor_cores(cin, cout, dtype):
    coords = scenes.shell32_batch(2)
    rng = np.random.default_rng(cin + cout)
    f = _rounded(scenes.normal_features(len(coords), cin, seed=cin), dtype)
    w = _rounded(scenes.conv_weight(cout, cin, 3, seed=cout), dtype)
    dout = _rounded(rng.standard_normal((len(coords), cout)), dtype)
    nbr = O.build_neighbor_map(coords, 3)
    dx, dw, db = _grads(_t(f, dtype), nbr, _t(w, dtype), _t(dout, dtype), True)
    rx, rw, rb = O.sparse_conv3d_grads(f, nbr, O.spconv_weight_to_kio(w), dout)
    assert max_rel_err(dx, rx) <= HALF_TOL
    assert max_rel_err(dw, rw) <= HALF_TOL
    assert max_rel_err(db, rb) <= HALF_TOL
    # the CUDA-core weight gradient gives the same result (fp32 accumulation both ways)
    _, dw_simt, _ = _grads(_t(f, dtype), nbr, _t(w, dtype), _t(dout, dtype), True,
                           algo=N.SV_CONV_SIMT)
    assert max_rel_err(dw, dw_simt) <= HALF_TOL


def test_tensor_core_weight_gradient_of_offsets_without_pairs():
    """Isolated voxels: only the centre offset has pairs, every other offset's gradient is an
    exact zero (items with an empty pair list still write their tile)."""

    coords = np.array([[0, 0, 0, 0], [0, 10, 10, 10], [1, 3, 4, 5], [1, -7, 2, 9]], np.int32)
    rng = np.random.default_rng(2)
    f = _t(rng.standard_normal((4, 64)), torch.bfloat16)
    dout = _t(rng.standard_normal((4, 128)), torch.bfloat16)
    nb = build_neighbor_map(_t(coords), 3)
    dw = conv3d_wgrad(f, dout, kmap_pairs(nb), (3, 3, 3), algo=N.SV_CONV_TCGEN05).float()
    dw = dw.reshape(128, 27, 64).cpu().numpy()
    assert np.count_nonzero(np.delete(dw, 13, axis=1)) == 0
    want = dout.float().cpu().numpy().T @ f.float().cpu().numpy()
    assert max_rel_err(dw[:, 13, :], want) <= HALF_TOL
    N.check_device_status(DEV)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_autograd_through_sparse_conv3d(dtype):
    coords = scenes.batched([scenes.shell(16, 5.5, 2.0, 1.0, seed=61),
                             scenes.shell(16, 6.0, 2.0, 1.0, seed=62)])
    cin, cout = 64, 128
    rng = np.random.default_rng(63)
    f = _rounded(scenes.normal_features(len(coords), cin, seed=64), dtype)
    w = _rounded(scenes.conv_weight(cout, cin, 3, seed=65), dtype)
    b = _rounded(0.1 * rng.standard_normal(cout), dtype)
    g = _rounded(rng.standard_normal((len(coords), cout)), dtype)
    conv = SparseConv3D(cin, cout, 3).to(DEV)
    conv.conv.weight = _t(w, dtype).requires_grad_(True)
    conv.conv.bias = _t(b, dtype).requires_grad_(True)
    feats = _t(f, dtype).requires_grad_(True)
    x = SparseTensor(feats, _t(coords))
    y = conv(x)
    assert y.features.requires_grad
    (y.features.float() * _t(g)).sum().backward()
    nbr = O.build_neighbor_map(coords, 3)
    ref_out = O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w), b)
    rx, rw, rb = O.sparse_conv3d_grads(f, nbr, O.spconv_weight_to_kio(w), g)
    tol = 1e-4 if dtype == torch.float32 else HALF_TOL
    assert max_rel_err(y.features.detach().float().cpu().numpy(), ref_out) <= tol
    assert max_rel_err(feats.grad.float().cpu().numpy(), rx) <= tol
    assert max_rel_err(_oki_to_kio_grad(conv.conv.weight.grad.float().cpu().numpy()), rw) <= tol
    assert max_rel_err(conv.conv.bias.grad.float().cpu().numpy(), rb) <= tol
    topo = MapTopology(x.cache, "3_1_(1, 1, 1)", x.cache["neighbors_3_1_(1, 1, 1)"])
    assert topo.unique() and "conv_pairs_3_1_(1, 1, 1)" in x.cache
    N.check_device_status(DEV)
