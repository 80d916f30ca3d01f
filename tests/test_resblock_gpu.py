"""The fused residual block on the GPU: the row-norm kernel against the oracle's LayerNorm32,
and SparseResBlock3D against the reference's own _SparseResBlock3D (fixtures, fp32) and against
the oracle in fp16 / bf16 at the SLat flow's I/O-block shapes."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mlx_diffuser_b200 import _native as N
from mlx_diffuser_b200 import scenes
from mlx_diffuser_b200.kernels.norm import row_norm
from mlx_diffuser_b200.layers.resblock import LayerNorm32, SparseResBlock3D
from mlx_diffuser_b200.layers.sparse import SparseTensor, sparse_downsample
from oracle import sparse_oracle as O
from tests.test_oracle import resblock_params

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _t(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def _rounded(a, dtype):
    return torch.from_numpy(np.asarray(a, np.float32)).to(dtype).float().numpy()


def max_rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


# ---- row norm --------------------------------------------------------------------------------


@pytest.mark.parametrize("channels", [8, 128, 130, 1024, 2048, 4096])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_row_norm_matches_layernorm32(channels, dtype):
    rng = np.random.default_rng(channels)
    coords = scenes.batched([scenes.shell(12, 4.0, 2.0, 0.5, seed=s) for s in range(3)])
    n = len(coords)
    x = _rounded(rng.standard_normal((n, channels)) * 3 + 1, dtype)
    w = (1 + 0.2 * rng.standard_normal(channels)).astype(np.float32)
    b = (0.2 * rng.standard_normal(channels)).astype(np.float32)
    scale = _rounded(0.3 * rng.standard_normal((3, channels)), dtype)
    shift = _rounded(0.3 * rng.standard_normal((3, channels)), dtype)
    xt = _t(x, dtype)
    tol = 2e-6 if dtype == torch.float32 else (4e-3 if dtype == torch.float16 else 8e-3)
    # affine + silu (norm1 of the block)
    got = row_norm(xt, weight=_t(w), bias=_t(b), silu=True).float().cpu().numpy()
    assert max_rel_err(got, O.silu(O.layernorm32(x, w, b))) <= tol
    # plain LayerNorm32 through the module
    got = LayerNorm32(channels, affine=False)(xt).float().cpu().numpy()
    assert max_rel_err(got, O.layernorm32(x)) <= tol
    # batch-indexed modulation + silu (norm2 of the block)
    got = row_norm(xt, scale=_t(scale, dtype), shift=_t(shift, dtype), coords=_t(coords, torch.int32),
                   batch_size=3, silu=True).float().cpu().numpy()
    bi = coords[:, 0]
    ref = O.silu(O.layernorm32(x) * (1 + scale[bi]) + shift[bi])
    assert max_rel_err(got, ref) <= tol
    # in place
    y = xt.clone()
    row_norm(y, weight=_t(w), bias=_t(b), out=y)
    assert max_rel_err(y.float().cpu().numpy(), O.layernorm32(x, w, b)) <= tol
    N.check_device_status(DEV)


@pytest.mark.parametrize("channels", [8, 64, 130, 1024])
def test_row_norm_strided_and_shared_modulation(channels):
    """scale / shift as the two halves of one [B, 2C] projection (row stride 2C, no copy) and
    as one row shared by every batch element (row stride 0)."""

    rng = np.random.default_rng(channels + 1)
    dtype = torch.bfloat16
    coords = scenes.batched([scenes.shell(12, 4.0, 2.0, 0.5, seed=s) for s in range(3)])
    x = _rounded(rng.standard_normal((len(coords), channels)), dtype)
    proj = _rounded(0.3 * rng.standard_normal((3, 2 * channels)), dtype)
    scale, shift = torch.chunk(_t(proj, dtype), 2, dim=-1)
    assert scale.stride(0) == 2 * channels
    ct = _t(coords, torch.int32)
    got = row_norm(_t(x, dtype), scale=scale, shift=shift, coords=ct, batch_size=3, silu=True)
    bi = coords[:, 0]
    ref = O.silu(O.layernorm32(x) * (1 + proj[bi, :channels]) + proj[bi, channels:])
    assert max_rel_err(got.float().cpu().numpy(), ref) <= 8e-3
    got = row_norm(_t(x, dtype), scale=scale[1:2], shift=shift[1], coords=ct, batch_size=3)
    ref = O.layernorm32(x) * (1 + proj[1, :channels]) + proj[1, channels:]
    assert max_rel_err(got.float().cpu().numpy(), ref) <= 8e-3
    N.check_device_status(DEV)


def test_row_norm_flags_bad_batch_index_and_rejects_bad_shapes():
    x = torch.randn((4, 16), device=DEV)
    coords = torch.tensor([[0, 0, 0, 0], [1, 0, 0, 1], [5, 0, 1, 0], [0, 1, 0, 0]],
                          dtype=torch.int32, device=DEV)
    row_norm(x, scale=torch.zeros((2, 16), device=DEV), coords=coords, batch_size=2)
    with pytest.raises(RuntimeError, match="out of range"):
        N.check_device_status(DEV)
    with pytest.raises(RuntimeError):  # odd channel count
        row_norm(torch.zeros((2, 7), device=DEV))
    with pytest.raises(ValueError, match="coordinates"):
        row_norm(x, shift=torch.zeros((2, 16), device=DEV))
    N.check_device_status(DEV)


# ---- residual block --------------------------------------------------------------------------


def _load_block(block: SparseResBlock3D, p: dict, dtype) -> SparseResBlock3D:
    block.norm1.weight = _t(p["norm1_w"])
    block.norm1.bias = _t(p["norm1_b"])
    block.conv1.conv.weight = _t(p["conv1_w"], dtype)
    block.conv1.conv.bias = _t(p["conv1_b"], dtype)
    block.conv2.conv.weight = _t(p["conv2_w"], dtype)
    block.conv2.conv.bias = _t(p["conv2_b"], dtype)
    lin = block.emb_layers[1]
    lin.weight.data = _t(p["emb_w"], dtype)
    lin.bias.data = _t(p["emb_b"], dtype)
    if "skip_w" in p:
        block.skip_connection.weight = _t(p["skip_w"], dtype)
        block.skip_connection.bias = _t(p["skip_b"], dtype)
    return block.to(DEV)


def test_resblock_matches_reference_fp32(resblock_golden):
    g = resblock_golden
    emb = _t(g["rb_emb"])
    x = SparseTensor(_t(g["rb_features"]), _t(g["rb_coords"], torch.int32))
    plain = _load_block(SparseResBlock3D(8, 12, out_channels=16), resblock_params(g, "plain"),
                        torch.float32)
    y = plain(x, emb)
    np.testing.assert_allclose(y.features.cpu().numpy(), g["plain_out"], rtol=1e-4, atol=1e-4)
    down = _load_block(SparseResBlock3D(16, 12, out_channels=16, downsample=True),
                       resblock_params(g, "down"), torch.float32)
    d = down(y, emb)
    assert np.array_equal(d.coords.cpu().numpy(), g["down_coords"])
    np.testing.assert_allclose(d.features.cpu().numpy(), g["down_out"], rtol=1e-4, atol=1e-4)
    up = _load_block(SparseResBlock3D(16, 12, out_channels=8, upsample=True),
                     resblock_params(g, "up"), torch.float32)
    u = up(d, emb)
    assert torch.equal(u.coords, x.coords)
    np.testing.assert_allclose(u.features.cpu().numpy(), g["up_out"], rtol=1e-4, atol=1e-4)
    N.check_device_status(DEV)


def _random_params(rng, cin, cout, emb_ch, dtype):
    p = {
        "norm1_w": (1 + 0.1 * rng.standard_normal(cin)).astype(np.float32),
        "norm1_b": (0.1 * rng.standard_normal(cin)).astype(np.float32),
        "conv1_w": _rounded(scenes.conv_weight(cout, cin, 3, int(rng.integers(1 << 30))), dtype),
        "conv1_b": _rounded(0.1 * rng.standard_normal(cout), dtype),
        "conv2_w": _rounded(scenes.conv_weight(cout, cout, 3, int(rng.integers(1 << 30))), dtype),
        "conv2_b": _rounded(0.1 * rng.standard_normal(cout), dtype),
        "emb_w": _rounded(rng.standard_normal((2 * cout, emb_ch)) / np.sqrt(emb_ch), dtype),
        "emb_b": _rounded(0.1 * rng.standard_normal(2 * cout), dtype),
    }
    if cin != cout:
        p["skip_w"] = _rounded(rng.standard_normal((cout, cin)) / np.sqrt(cin), dtype)
        p["skip_b"] = _rounded(0.1 * rng.standard_normal(cout), dtype)
    return p


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_resblock_io_shapes_half_vs_oracle(dtype):
    """The SLat flow's input blocks at 64^3: ResBlock(128 -> 128), then the downsampling
    ResBlock(128 -> 1024) -- conv 128 -> 1024 and 1024 -> 1024 at 32^3 on tensor cores."""

    rng = np.random.default_rng(7)
    coords = scenes.batched([scenes.shell64(11), scenes.shell64(12)])
    x0 = _rounded(rng.standard_normal((len(coords), 128)), dtype)
    emb = _rounded(rng.standard_normal((2, 256)), dtype)
    p1 = _random_params(rng, 128, 128, 256, dtype)
    p2 = _random_params(rng, 128, 1024, 256, dtype)
    b1 = _load_block(SparseResBlock3D(128, 256), p1, dtype)
    b2 = _load_block(SparseResBlock3D(128, 256, out_channels=1024, downsample=True), p2, dtype)
    x = SparseTensor(_t(x0, dtype), _t(coords, torch.int32))
    y = b1(x, _t(emb, dtype))
    z = b2(y, _t(emb, dtype))
    N.check_device_status(DEV)
    # oracle in fp32 on the same rounded inputs; the second block starts from the GPU's first
    # block output so each block is checked against its own input
    r1 = O.resblock(coords, x0, emb, p1)
    assert max_rel_err(y.features.float().cpu().numpy(), r1) <= 1e-2
    y_np = y.features.float().cpu().numpy()
    dc, inv = O.downsample_coords(coords, 2)
    assert np.array_equal(z.coords.cpu().numpy(), dc)
    pooled = _rounded(O.downsample_features(y_np, inv, len(dc)), dtype)
    r2 = O.resblock(dc, pooled, emb, p2)
    assert max_rel_err(z.features.float().cpu().numpy(), r2) <= 1e-2


def test_captured_resblock_stack_replays_bit_exactly():
    """The I/O stack (with a downsample and an upsample) captured in a CUDA graph gives the same
    bits as the eager run, for new input values, and the downsample's coordinates are reused."""

    from mlx_diffuser_b200.graphs import CapturedForward

    rng = np.random.default_rng(3)
    dtype = torch.float16
    coords = _t(scenes.batched([scenes.shell64(31), scenes.shell64(32)]), torch.int32)
    n = coords.shape[0]
    blocks = []
    for cin, cout, kw in ((128, 128, {}), (128, 256, {"downsample": True}),
                          (256, 128, {"upsample": True})):
        blocks.append(_load_block(SparseResBlock3D(cin, 64, out_channels=cout, **kw),
                                  _random_params(rng, cin, cout, 64, dtype), dtype))
    probe = SparseTensor(torch.zeros((n, 128), device=DEV, dtype=dtype), coords)
    cache, batch, spatial = probe.cache, probe.batch_size, probe.spatial_shape

    def stack(feats, emb):
        h = SparseTensor(feats, coords, batch, spatial, (1, 1, 1), cache)
        for b in blocks:
            h = b(h, emb)
        return h.features

    graphed = CapturedForward(stack)
    for seed in (0, 1):
        f = torch.from_numpy(rng.standard_normal((n, 128))).to(DEV, dtype)
        e = torch.from_numpy(rng.standard_normal((2, 64))).to(DEV, dtype)
        eager = stack(f, e).clone()
        replayed = graphed(f, e).clone()
        assert torch.equal(eager, replayed), seed
    assert f"downsample_coords_2_{(1, 1, 1)}" in cache
    N.check_device_status(DEV)
    graphed.release()

