"""Pin the CPU oracle against fixtures produced by the reference's own sparse-voxel code.

The fixtures under ``tests/golden`` were made by ``tests/golden/make_golden.py``, which runs
mlx_diffuser's ``layers/sparse.py`` and ``kernels/sparse.py`` unmodified (fallback conv path).
Integer outputs must match bit-exactly; float32 features to float32 summation-order noise.
"""

from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import sparse_oracle as O
from tests.conftest import load_golden


def _maps(g):
    yield int(g["kernel_size"]), int(g["dilation"]), g["nbr"]
    i = 0
    while f"nbr_extra{i}" in g:
        yield tuple(g[f"nbr_extra{i}_kernel"]), tuple(g[f"nbr_extra{i}_dilation"]), g[f"nbr_extra{i}"]
        i += 1


def test_kernel_map_bit_exact(golden):
    _, g = golden
    for ks, dl, want in _maps(g):
        ks = ks if isinstance(ks, int) else tuple(int(v) for v in ks)
        dl = dl if isinstance(dl, int) else tuple(int(v) for v in dl)
        assert np.array_equal(O.build_neighbor_map(g["coords"], ks, dl), want)
        if len(g["coords"]) <= 2500:
            assert np.array_equal(O.build_neighbor_map_dict(g["coords"], ks, dl), want)


def test_conv_matches_reference_fallback(golden):
    _, g = golden
    w = O.spconv_weight_to_kio(g["weight"])
    got = O.sparse_conv3d(g["features"], g["nbr"], w, g["bias"])
    np.testing.assert_allclose(got, g["conv_out"], rtol=1e-5, atol=1e-5)


def test_downsample_upsample_bit_exact(golden):
    _, g = golden
    factors = sorted(int(k[4:-7]) for k in g if k.startswith("down") and k.endswith("_coords"))
    assert factors
    for f in factors:
        coords, inverse = O.downsample_coords(g["coords"], f)
        assert np.array_equal(coords, g[f"down{f}_coords"])
        assert np.array_equal(inverse, g[f"down{f}_inverse"])
        pooled = O.downsample_features(g["features"], inverse, len(coords))
        # np.add.at sums in row order, exactly like the reference's scatter-add
        assert np.array_equal(pooled, g[f"down{f}_features"])
        assert np.array_equal(O.upsample_features(pooled, inverse), g[f"up{f}_features"])
        shape = O.downsample_spatial_shape(tuple(g["spatial_shape"]), f)
        assert shape == tuple(g[f"down{f}_spatial_shape"])


def test_reference_block_pool_divides_by_count_plus_one():
    """``tests/test_trellis.py:147-161`` of the reference: a 2^3 block pools to sum / 9."""

    g = load_golden("ref_test_block2")
    assert g["down2_coords"].shape == (1, 4)
    np.testing.assert_allclose(g["up2_features"], np.broadcast_to(g["features"].sum(0) / 9, (8, 2)))


def test_offsets_order_matches_reference():
    offs = O.kernel_offsets(3)
    assert len(offs) == 27 and offs[0] == (-1, -1, -1) and offs[13] == (0, 0, 0)
    assert offs[1] == (-1, -1, 0) and offs[9] == (0, -1, -1)
    with pytest.raises(ValueError):
        O.kernel_offsets(4)


REF = os.environ.get("MLX_DIFFUSER_REF", "/root/reference")


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "src", "mlx_diffuser")),
                    reason="reference sources not present")
def test_oracle_against_live_reference_random_cases():
    """Where the reference sources exist, run them under the NumPy shim on fresh random
    inputs (duplicates, negatives, several batches) and compare with the oracle."""

    from tests.golden.make_golden import load_reference, run_case

    ref = load_reference(REF)
    rng = np.random.default_rng(99)
    for _ in range(3):
        n = int(rng.integers(1, 300))
        c = rng.integers(-4, 5, size=(n, 4)).astype(np.int32)
        c[:, 0] = rng.integers(0, 3, size=n)
        feats = rng.standard_normal((n, 3)).astype(np.float32)
        w = rng.standard_normal((2, 3, 3, 3, 3)).astype(np.float32)
        b = rng.standard_normal(2).astype(np.float32)
        g = run_case(ref, c, feats, w, b, factors=(2, 4))
        assert np.array_equal(O.build_neighbor_map(c, 3), g["nbr"])
        np.testing.assert_allclose(
            O.sparse_conv3d(feats, g["nbr"], O.spconv_weight_to_kio(w), b), g["conv_out"],
            rtol=1e-5, atol=1e-5)
        for f in (2, 4):
            coords, inverse = O.downsample_coords(c, f)
            assert np.array_equal(coords, g[f"down{f}_coords"])
            assert np.array_equal(inverse, g[f"down{f}_inverse"])


# ---- topology: subdivide, attention windows, occupancy -------------------------------------


def _groups_as_perm(groups):
    return np.concatenate(groups), np.cumsum([0] + [len(g) for g in groups])


def test_subdivide_matches_reference(topology_golden):
    g = topology_golden
    coords, feats = O.subdivide(g["sub_coords_in"], g["sub_features_in"])
    assert np.array_equal(coords, g["sub_coords"])
    assert np.array_equal(feats, g["sub_features"])


def test_attention_groups_match_reference(topology_golden):
    g = topology_golden
    i = 0
    while f"win{i}_perm" in g:
        window = int(g[f"win{i}_window"])
        groups = O.attention_groups(g["win_coords"], None if window < 0 else window,
                                    tuple(int(v) for v in g[f"win{i}_shift"]))
        perm, offsets = _groups_as_perm(groups)
        assert np.array_equal(perm, g[f"win{i}_perm"])
        assert np.array_equal(offsets, g[f"win{i}_offsets"])
        i += 1
    assert i == 4


def test_occupied_coordinates_match_reference(topology_golden):
    g = topology_golden
    for i in range(3):
        got = O.occupied_coordinates(g["occ_logits"], float(g[f"occ{i}_threshold"]))
        assert np.array_equal(got, g[f"occ{i}_coords"])
    half = g["occ_half_logits"]
    got = O.occupied_coordinates(half.astype(np.float32), float(g["occ_half_threshold"]),
                                 "float16")
    assert np.array_equal(got, g["occ_half_coords"])
    # float16(0.3) > 0.3 and one logit equals it: a comparison against the unrounded
    # threshold would list that cell
    unrounded = np.argwhere(half.astype(np.float64) > float(g["occ_half_threshold"]))
    assert len(unrounded) == len(g["occ_half_coords"]) + 1


# ---- residual block --------------------------------------------------------------------------


def resblock_params(g, prefix):
    keys = ("norm1_w", "norm1_b", "conv1_w", "conv1_b", "conv2_w", "conv2_b", "emb_w", "emb_b",
            "skip_w", "skip_b")
    return {k: g[f"{prefix}_{k}"] for k in keys if f"{prefix}_{k}" in g}


def test_resblock_matches_reference(resblock_golden):
    g = resblock_golden
    coords, feats, emb = g["rb_coords"], g["rb_features"], g["rb_emb"]
    y = O.resblock(coords, feats, emb, resblock_params(g, "plain"))
    np.testing.assert_allclose(y, g["plain_out"], rtol=1e-4, atol=1e-4)
    # downsample block: pooled features of the plain block's output, on the coarse coords
    dc, inv = O.downsample_coords(coords, 2)
    assert np.array_equal(dc, g["down_coords"])
    pooled = O.downsample_features(g["plain_out"], inv, len(dc))
    d = O.resblock(dc, pooled, emb, resblock_params(g, "down"))
    np.testing.assert_allclose(d, g["down_out"], rtol=1e-4, atol=1e-4)
    # upsample block: the coarse output gathered back to the fine coords
    u = O.resblock(coords, O.upsample_features(g["down_out"], inv), emb, resblock_params(g, "up"))
    np.testing.assert_allclose(u, g["up_out"], rtol=1e-4, atol=1e-4)


# ---- gradients ----------------------------------------------------------------------------------


def test_gradient_oracle_matches_autograd_of_the_fallback(golden):
    """The closed-form gradients equal torch autograd (float64) of the reference's fallback
    formula, out = bias + sum_k (features[max(nbr, 0)] @ W[k]) * valid, duplicates included."""

    import torch

    name, g = golden
    if len(g["coords"]) > 2500:
        pytest.skip("small fixtures only")
    nbr = g["nbr"]
    w = O.spconv_weight_to_kio(g["weight"]).astype(np.float64)
    f = torch.tensor(g["features"], dtype=torch.float64, requires_grad=True)
    wt = torch.tensor(w, requires_grad=True)
    b = torch.tensor(g["bias"], dtype=torch.float64, requires_grad=True)
    nb = torch.from_numpy(nbr.astype(np.int64))
    out = b.expand(len(nbr), -1)
    for k in range(nbr.shape[1]):
        valid = (nb[:, k] >= 0).to(torch.float64)[:, None]
        out = out + (f[nb[:, k].clamp(min=0)] @ wt[k]) * valid
    dout = np.random.default_rng(4).standard_normal(out.shape)
    out.backward(torch.from_numpy(dout))
    dx, dw, db = O.sparse_conv3d_grads(g["features"], nbr, w, dout, accum=np.float64)
    np.testing.assert_allclose(dx, f.grad.numpy(), rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(dw, wt.grad.numpy(), rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(db, b.grad.numpy(), rtol=1e-10, atol=1e-10)


def test_vectorised_map_agrees_with_dict_map_for_large_batch_indices():
    """The packed-key fast path keeps 4 bits for the batch index; larger indices take the dict
    path (a guard that once let batch indices up to 2^20 into the 64-bit key collided)."""

    rng = np.random.default_rng(3)
    c = rng.integers(0, 6, size=(300, 4)).astype(np.int32)
    for scale in (1, 5, 100000):
        cc = c.copy()
        cc[:, 0] = rng.integers(0, 4, size=300) * scale
        assert np.array_equal(O.build_neighbor_map(cc, 3), O.build_neighbor_map_dict(cc, 3))
