"""Sparse convolution on the GPU against the reference's fallback (fp32 oracle).

Tolerances, from the path's contract:
* fp32 features: within rtol 1e-4 of the fp32 reference (plus an absolute floor of
  1e-4 x max|ref| for outputs near zero);
* fp16 / bf16 features: max relative error <= 1e-2 of the fp32 reference, where
  max relative error = max|out - ref| / max|ref| and the reference is computed in fp32 from
  the same (rounded) inputs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mlx_diffuser_b200 import _native as N
from mlx_diffuser_b200 import scenes
from mlx_diffuser_b200.kernels.sparse import conv3d_forward, sparse_conv3d
from mlx_diffuser_b200.layers.sparse import (
    SparseConv3D,
    SparseTensor,
    build_neighbor_map,
    conv_row_order,
)
from oracle import sparse_oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
HALF_TOL = 1e-2
F32_RTOL = 1e-4


def max_rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / scale)


def assert_f32_close(got, ref):
    ref = np.asarray(ref, np.float64)
    np.testing.assert_allclose(got, ref, rtol=F32_RTOL, atol=F32_RTOL * max(np.abs(ref).max(), 1e-6))


def _module(weight, bias, dtype, dilation=1, algo=N.SV_CONV_AUTO):
    o, k, _, _, i = weight.shape
    conv = SparseConv3D(i, o, k, dilation=dilation).to(DEV)
    conv.conv.weight = torch.from_numpy(weight).to(DEV, dtype)
    conv.conv.bias = torch.from_numpy(bias).to(DEV, dtype)
    conv.algo = algo
    return conv


def _run(coords, feats, weight, bias, dtype, dilation=1, algo=N.SV_CONV_AUTO):
    conv = _module(weight, bias, dtype, dilation, algo)
    x = SparseTensor(torch.from_numpy(feats).to(DEV, dtype), torch.from_numpy(coords).to(DEV))
    out = conv(x).features.float().cpu().numpy()
    N.check_device_status(DEV)
    return out, x


def _rounded(a, dtype):
    return torch.from_numpy(np.asarray(a, np.float32)).to(dtype).float().numpy()


def test_conv_fp32_matches_golden(golden):
    _, g = golden
    out, _ = _run(g["coords"], g["features"], g["weight"], g["bias"], torch.float32,
                  int(g["dilation"]))
    assert_f32_close(out, g["conv_out"])


def test_reference_metal_kernel_equals_fallback_four_points():
    """``tests/test_trellis.py:119-131`` of the reference, against its recorded output."""

    from tests.conftest import load_golden

    g = load_golden("ref_test_four_points")
    out, _ = _run(g["coords"], g["features"], g["weight"], g["bias"], torch.float32)
    np.testing.assert_allclose(out, g["conv_out"], atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("algo", [N.SV_CONV_AUTO, N.SV_CONV_SIMT])
def test_conv_half_matches_fp32_reference(golden, dtype, algo):
    _, g = golden
    f = _rounded(g["features"], dtype)
    w = _rounded(g["weight"], dtype)
    b = _rounded(g["bias"], dtype)
    ref = O.sparse_conv3d(f, g["nbr"], O.spconv_weight_to_kio(w), b)
    out, _ = _run(g["coords"], f, w, b, dtype, int(g["dilation"]), algo)
    assert max_rel_err(out, ref) <= HALF_TOL


@pytest.mark.parametrize(
    "cin,cout",
    [(64, 32), (64, 64), (128, 128), (64, 256), (192, 512), (1024, 1024), (256, 96),
     # Cin an odd multiple of 32: 32-channel K stages with the 64-byte swizzle
     (32, 32), (32, 128), (96, 64), (160, 256)],
)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tcgen05_shapes(cin, cout, dtype):
    coords = scenes.batched(
        [scenes.shell(16, 5.5, 2.0, 1.0, seed=7), scenes.shell(12, 4.0, 2.0, 0.5, seed=9)]
    )
    f = _rounded(scenes.normal_features(len(coords), cin, seed=1), dtype)
    w = _rounded(scenes.conv_weight(cout, cin, 3, seed=2), dtype)
    b = _rounded(np.random.default_rng(3).standard_normal(cout).astype(np.float32) * 0.1, dtype)
    nbr = O.build_neighbor_map(coords, 3)
    ref = O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w), b)
    out, _ = _run(coords, f, w, b, dtype, algo=N.SV_CONV_TCGEN05)
    assert max_rel_err(out, ref) <= HALF_TOL


@pytest.mark.parametrize("cin,cout", [(8, 128), (16, 64), (128, 8), (64, 16), (8, 8), (16, 16),
                                      (8, 32), (256, 8)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tcgen05_small_channels(cin, cout, dtype):
    """8 or 16 channels on the tensor cores: 32 / Cin offsets packed into one K stage, N = 16
    tiles for 8 or 16 outputs (the I/O convolutions of the SLat stack)."""

    coords = scenes.batched(
        [scenes.shell(16, 5.5, 2.0, 1.0, seed=7), scenes.shell(12, 4.0, 2.0, 0.5, seed=9)]
    )
    f = _rounded(scenes.normal_features(len(coords), cin, seed=1), dtype)
    w = _rounded(scenes.conv_weight(cout, cin, 3, seed=2), dtype)
    b = _rounded(np.random.default_rng(3).standard_normal(cout).astype(np.float32) * 0.1, dtype)
    nbr = O.build_neighbor_map(coords, 3)
    ref = O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w), b)
    out, x = _run(coords, f, w, b, dtype, algo=N.SV_CONV_TCGEN05)
    assert max_rel_err(out, ref) <= HALF_TOL
    # with a residual added in the epilogue
    nbr_d = x.cache["neighbors_3_1_(1, 1, 1)"]
    res = _rounded(scenes.normal_features(len(coords), cout, seed=4), dtype)
    got = conv3d_forward(x.features, nbr_d, torch.from_numpy(w).to(DEV, dtype).contiguous(),
                         N.SV_WEIGHT_OKI, torch.from_numpy(b).to(DEV, dtype), cout,
                         algo=N.SV_CONV_TCGEN05, residual=torch.from_numpy(res).to(DEV, dtype))
    assert max_rel_err(got.float().cpu().numpy(), ref + res) <= HALF_TOL
    N.check_device_status(DEV)


def test_tcgen05_packed_offsets_past_the_kernel_volume():
    """A 3 x 1 x 3 kernel (9 offsets) at 8 input channels: the third group of 4 packed offsets
    holds offset 8 and three that do not exist, which must contribute nothing."""

    coords = scenes.shell(16, 5.5, 2.0, 1.0, seed=5)
    dtype = torch.bfloat16
    c = torch.from_numpy(coords).to(DEV)
    nbr = build_neighbor_map(c, (3, 1, 3))
    f = _rounded(scenes.normal_features(len(coords), 8, seed=6), dtype)
    w = _rounded(np.random.default_rng(7).standard_normal((64, 9, 8)) / np.sqrt(72), dtype)
    ref = O.sparse_conv3d(f, nbr.cpu().numpy(), np.ascontiguousarray(w.transpose(1, 2, 0)),
                          np.zeros(64, np.float32))
    out = conv3d_forward(torch.from_numpy(f).to(DEV, dtype), nbr,
                         torch.from_numpy(w).to(DEV, dtype).contiguous(), N.SV_WEIGHT_OKI, None, 64,
                         algo=N.SV_CONV_TCGEN05)
    N.check_device_status(DEV)
    assert max_rel_err(out.float().cpu().numpy(), ref) <= HALF_TOL


@pytest.mark.parametrize("cin,cout", [(32, 32), (64, 96), (128, 128), (96, 64), (160, 256),
                                      (256, 32)])
def test_tf32x3_fp32_shapes(cin, cout):
    """fp32 on the tensor cores (3xTF32) against the oracle at rtol 1e-4, with bias, in both
    weight layouts, and with a residual. Against a float64 evaluation its max relative error stays
    below 3e-5 (the CUDA-core fp32 kernel measures ~1e-6 to 1.5e-5 on these shapes; 3xTF32 drops
    the lo x lo products, ~2^-20 of each product)."""

    coords = scenes.batched(
        [scenes.shell(16, 5.5, 2.0, 1.0, seed=7), scenes.shell(12, 4.0, 2.0, 0.5, seed=9)]
    )
    f = scenes.normal_features(len(coords), cin, seed=1)
    w = scenes.conv_weight(cout, cin, 3, seed=2)
    b = (np.random.default_rng(3).standard_normal(cout) * 0.1).astype(np.float32)
    nbr = O.build_neighbor_map(coords, 3)
    ref = O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w), b, accum=np.float64)
    out, x = _run(coords, f, w, b, torch.float32, algo=N.SV_CONV_TCGEN05)
    assert_f32_close(out, ref)
    assert max_rel_err(out, ref) <= 3e-5
    simt, _ = _run(coords, f, w, b, torch.float32, algo=N.SV_CONV_SIMT)
    assert_f32_close(simt, ref)
    # the functional form with a (K, Cin, Cout) weight, and a residual added in the epilogue
    nbr_d = x.cache["neighbors_3_1_(1, 1, 1)"]
    feats = torch.from_numpy(f).to(DEV)
    wk = torch.from_numpy(O.spconv_weight_to_kio(w)).to(DEV).contiguous()
    fun = conv3d_forward(feats, nbr_d, wk, N.SV_WEIGHT_KIO, torch.from_numpy(b).to(DEV), cout,
                         algo=N.SV_CONV_TCGEN05)
    assert_f32_close(fun.cpu().numpy(), ref)
    res = torch.from_numpy(scenes.normal_features(len(coords), cout, seed=4)).to(DEV)
    wo = torch.from_numpy(w).to(DEV).contiguous()
    with_res = conv3d_forward(feats, nbr_d, wo, N.SV_WEIGHT_OKI, torch.from_numpy(b).to(DEV),
                              cout, algo=N.SV_CONV_TCGEN05, residual=res)
    assert_f32_close(with_res.cpu().numpy(), ref + res.cpu().numpy())
    N.check_device_status(DEV)


def test_tf32x3_config1_every_row():
    """Config 1 (64^3 shell, ~20k rows, 128 -> 128, fp32) on the 3xTF32 kernel: every row
    against the fp32 oracle at rtol 1e-4, several persistent work items per CTA."""

    coords = scenes.shell64(0)
    f = scenes.normal_features(len(coords), 128, seed=1)
    w = scenes.conv_weight(128, 128, 3, seed=2)
    b = np.zeros(128, np.float32)
    out, x = _run(coords, f, w, b, torch.float32, algo=N.SV_CONV_TCGEN05)
    nbr = x.cache["neighbors_3_1_(1, 1, 1)"].cpu().numpy()
    assert np.array_equal(nbr, O.build_neighbor_map(coords, 3))
    assert_f32_close(out, O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w), b, accum=np.float64))


@pytest.mark.parametrize("cin,cout", [(64, 64), (64, 128), (64, 256), (32, 32), (32, 256)])
def test_tcgen05_persistent_ctas_take_several_items(cin, cout):
    """24k rows give more work items than SMs, so each persistent CTA runs several items and
    reuses both accumulator buffers and both work slots; every item must match the reference."""

    coords = scenes.shell32_batch(4)
    dtype = torch.bfloat16
    f = _rounded(scenes.normal_features(len(coords), cin, seed=31), dtype)
    w = _rounded(scenes.conv_weight(cout, cin, 3, seed=32), dtype)
    b = _rounded(np.random.default_rng(33).standard_normal(cout).astype(np.float32), dtype)
    ref = O.sparse_conv3d(f, O.build_neighbor_map(coords, 3), O.spconv_weight_to_kio(w), b)
    out, _ = _run(coords, f, w, b, dtype, algo=N.SV_CONV_TCGEN05)
    assert max_rel_err(out, ref) <= HALF_TOL


def test_tcgen05_agrees_with_simt_and_ignores_row_order():
    coords = scenes.shell32_batch(2)
    cin = cout = 128
    dtype = torch.bfloat16
    feats = torch.from_numpy(scenes.normal_features(len(coords), cin, seed=5)).to(DEV, dtype)
    w = torch.from_numpy(scenes.conv_weight(cout, cin, 3, seed=6)).to(DEV, dtype).contiguous()
    b = torch.zeros(cout, device=DEV, dtype=dtype)
    nbr = build_neighbor_map(torch.from_numpy(coords).to(DEV), 3)
    order, tiles = conv_row_order(nbr)
    tc_plain = conv3d_forward(feats, nbr, w, N.SV_WEIGHT_OKI, b, cout, algo=N.SV_CONV_TCGEN05)
    tc_order = conv3d_forward(feats, nbr, w, N.SV_WEIGHT_OKI, b, cout, row_order=order,
                              tile_order=tiles, algo=N.SV_CONV_TCGEN05)
    simt = conv3d_forward(feats, nbr, w, N.SV_WEIGHT_OKI, b, cout, row_order=order,
                          algo=N.SV_CONV_SIMT)
    N.check_device_status(DEV)
    assert max_rel_err(tc_plain.float().cpu(), tc_order.float().cpu()) <= 1e-6
    assert max_rel_err(tc_order.float().cpu(), simt.float().cpu()) <= HALF_TOL


def test_functional_kio_matches_module_oki():
    coords = scenes.shell(16, 5.5, 2.0, 1.0, seed=11)
    for dtype, cin, cout in ((torch.bfloat16, 64, 64), (torch.float32, 16, 24)):
        f = scenes.normal_features(len(coords), cin, seed=12)
        w = scenes.conv_weight(cout, cin, 3, seed=13)
        b = np.random.default_rng(14).standard_normal(cout).astype(np.float32)
        mod, x = _run(coords, f, w, b, dtype)
        nbr = x.cache["neighbors_3_1_(1, 1, 1)"]
        fun = sparse_conv3d(
            x.features, nbr, torch.from_numpy(O.spconv_weight_to_kio(w)).to(DEV, dtype),
            torch.from_numpy(b).to(DEV, dtype),
        )
        assert fun.dtype == dtype
        assert max_rel_err(fun.float().cpu(), mod) <= (1e-6 if dtype == torch.float32 else 1e-2)


def test_config2_full_size_every_row():
    """4 x ~6k-voxel shells at 32^3, 1024 -> 1024, bf16 (the benchmark's workload): every one
    of the 24,168 output rows against the fp32 oracle (about 1 TFLOP of host BLAS)."""

    coords = scenes.shell32_batch(4)
    dtype = torch.bfloat16
    f = _rounded(scenes.normal_features(len(coords), 1024, seed=21), dtype)
    w = _rounded(scenes.conv_weight(1024, 1024, 3, seed=22), dtype)
    b = _rounded(np.random.default_rng(23).standard_normal(1024) * 0.1, dtype)
    out, x = _run(coords, f, w, b, dtype)
    nbr = x.cache["neighbors_3_1_(1, 1, 1)"].cpu().numpy()
    assert np.array_equal(nbr, O.build_neighbor_map(coords, 3))
    ref = O.sparse_conv3d(f, nbr, O.spconv_weight_to_kio(w), b)
    assert out.shape == ref.shape == (len(coords), 1024)
    assert max_rel_err(out, ref) <= HALF_TOL


def test_conv_edge_cases():
    dtype = torch.bfloat16
    cin = cout = 64
    w = torch.from_numpy(scenes.conv_weight(cout, cin, 3, seed=1)).to(DEV, dtype).contiguous()
    bias = torch.linspace(-1, 1, cout, device=DEV).to(dtype)
    for algo in (N.SV_CONV_TCGEN05, N.SV_CONV_SIMT):
        # all neighbours missing -> bias only
        feats = torch.randn(5, cin, device=DEV).to(dtype)
        nbr = torch.full((5, 27), -1, dtype=torch.int32, device=DEV)
        out = conv3d_forward(feats, nbr, w, N.SV_WEIGHT_OKI, bias, cout, algo=algo)
        assert torch.equal(out, bias.expand(5, cout))
        # out-of-range neighbour indices are flagged and treated as missing
        nbr[:, 0] = 99
        out = conv3d_forward(feats, nbr, w, N.SV_WEIGHT_OKI, bias, cout, algo=algo)
        assert torch.equal(out, bias.expand(5, cout))
        with pytest.raises(RuntimeError, match="out of range"):
            N.check_device_status(DEV)
    # partial tiles: N = 1, 127, 129, 257
    for n in (1, 127, 129, 257):
        coords = scenes.shell(16, 5.5, 2.0, 1.0, seed=3)[:n]
        f = _rounded(scenes.normal_features(n, cin, seed=n), dtype)
        wn = _rounded(scenes.conv_weight(cout, cin, 3, seed=4), dtype)
        out, _ = _run(coords, f, wn, np.zeros(cout, np.float32), dtype)
        ref = O.sparse_conv3d(f, O.build_neighbor_map(coords, 3), O.spconv_weight_to_kio(wn),
                              np.zeros(cout, np.float32))
        assert max_rel_err(out, ref) <= HALF_TOL
    # empty input and zero output channels
    empty = SparseTensor(torch.zeros((0, cin), device=DEV, dtype=dtype),
                         torch.zeros((0, 4), dtype=torch.int32, device=DEV))
    conv = SparseConv3D(cin, cout).to(DEV)
    conv.cast_dtype(dtype)
    assert conv(empty).features.shape == (0, cout)
    zero_out = sparse_conv3d(torch.zeros((3, cin), device=DEV), torch.zeros((3, 27), dtype=torch.int32),
                             torch.zeros((27, cin, 0)), torch.zeros(0))
    assert zero_out.shape == (3, 0)


@pytest.mark.parametrize("algo", [N.SV_CONV_TCGEN05, N.SV_CONV_SIMT])
def test_row_subset_conv_matches_full_conv_and_leaves_other_rows(algo):
    """``rows=`` computes exactly those output rows (the halo overlap's interior and boundary
    passes) with their own schedule, and leaves every other row of ``out`` untouched."""

    from mlx_diffuser_b200.kernels.sparse import conv3d_forward
    from mlx_diffuser_b200.layers.sparse import build_neighbor_map, conv_row_order

    coords = scenes.shell32_batch(2)
    dtype = torch.bfloat16
    f = torch.from_numpy(scenes.normal_features(len(coords), 64, seed=5)).to(DEV, dtype)
    w = torch.from_numpy(scenes.conv_weight(128, 64, 3, seed=6)).to(DEV, dtype).contiguous()
    b = torch.linspace(-1, 1, 128, device=DEV).to(dtype)
    nbr = build_neighbor_map(torch.from_numpy(coords).to(DEV), 3)
    ro, to = conv_row_order(nbr)
    full = conv3d_forward(f, nbr, w, N.SV_WEIGHT_OKI, b, 128, row_order=ro, tile_order=to,
                          algo=algo)
    subset = torch.from_numpy(np.random.default_rng(1).choice(len(coords), 5000,
                                                              replace=False)).to(DEV)
    sro, sto = conv_row_order(nbr[subset].contiguous())
    rows = subset[sro.long()].to(torch.int32)
    out = torch.full_like(full, 7.0)
    conv3d_forward(f, nbr, w, N.SV_WEIGHT_OKI, b, 128, rows=rows, tile_order=sto, out=out,
                   algo=algo)
    assert torch.equal(out[subset], full[subset])
    mask = torch.ones(len(coords), dtype=torch.bool, device=DEV)
    mask[subset] = False
    assert bool((out[mask] == 7.0).all())
    N.check_device_status(DEV)


def _fused_halo_case():
    from mlx_diffuser_b200.layers.sparse import build_neighbor_map, conv_row_order

    coords = scenes.shell32_batch(2)
    n = len(coords)
    f = torch.from_numpy(scenes.normal_features(n, 64, seed=8)).to(DEV, torch.bfloat16)
    w = torch.from_numpy(scenes.conv_weight(64, 64, 3, seed=9)).to(DEV, torch.bfloat16).contiguous()
    b = torch.linspace(-1, 1, 64, device=DEV).to(torch.bfloat16)
    nbr = build_neighbor_map(torch.from_numpy(coords).to(DEV), 3)
    perm = torch.from_numpy(np.random.default_rng(2).permutation(n)).to(DEV)
    first, second = perm[: n // 3 * 2], perm[n // 3 * 2:]
    segs = []
    for sub in (first, second):
        ro, to = conv_row_order(nbr[sub].contiguous())
        segs.append((sub[ro.long()].to(torch.int32), to))
    n_in = (segs[0][0].numel() + 127) // 128
    pad = torch.full((n_in * 128 - segs[0][0].numel(),), -1, dtype=torch.int32, device=DEV)
    rows = torch.cat([segs[0][0], pad, segs[1][0]])
    tiles = torch.cat([segs[0][1], segs[1][1] + n_in]).to(torch.int32)
    return f, nbr, w, b, rows, tiles, n_in


def test_fused_halo_conv_with_raised_flag_matches_full_conv():
    """One launch over [interior rows; padding; boundary rows] whose boundary tiles wait for a
    data flag that is already raised: same output as the plain convolution."""

    import ctypes

    from mlx_diffuser_b200.kernels.sparse import conv3d_forward, conv3d_forward_halo

    f, nbr, w, b, rows, tiles, n_in = _fused_halo_case()
    full = conv3d_forward(f, nbr, w, N.SV_WEIGHT_OKI, b, 64)
    flag = torch.full((1,), 5, dtype=torch.int64, device=DEV)
    flags = (ctypes.c_void_p * 8)(flag.data_ptr())
    out = torch.full_like(full, 3.0)
    conv3d_forward_halo(f, nbr, w, b, 64, rows, tiles, n_in, flags, 1, 5, out=out)
    assert torch.equal(out, full)
    N.check_device_status(DEV)


def test_fused_halo_conv_reports_an_expired_wait_and_stays_usable():
    """A data flag that nothing raises: every waiting CTA gives up after its bounded wait, the
    launch completes, the status word carries SV_DEVICE_WAIT_TIMEOUT, and the context keeps
    working (a plain convolution afterwards is correct)."""

    import ctypes

    from mlx_diffuser_b200.kernels.sparse import conv3d_forward, conv3d_forward_halo

    f, nbr, w, b, rows, tiles, n_in = _fused_halo_case()
    flag = torch.zeros((1,), dtype=torch.int64, device=DEV)
    flags = (ctypes.c_void_p * 8)(flag.data_ptr())
    out = torch.empty((f.shape[0], 64), dtype=f.dtype, device=DEV)
    conv3d_forward_halo(f, nbr, w, b, 64, rows, tiles, n_in, flags, 1, 1, out=out)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="timed out"):
        N.check_device_status(DEV)
    full = conv3d_forward(f, nbr, w, N.SV_WEIGHT_OKI, b, 64)
    ref = conv3d_forward(f, nbr, w, N.SV_WEIGHT_OKI, b, 64, algo=N.SV_CONV_SIMT)
    assert max_rel_err(full.float().cpu().numpy(), ref.float().cpu().numpy()) <= HALF_TOL
    N.check_device_status(DEV)
