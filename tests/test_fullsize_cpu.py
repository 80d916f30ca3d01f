"""The full-size checks of ``tests/fullsize.py`` themselves, on CPU tensors: they pass the
oracle's own output and catch a single wrong row or a wrong offset weight."""

from __future__ import annotations

import numpy as np
import torch

from mlx_diffuser_b200 import scenes
from oracle import sparse_oracle as O
from tests.fullsize import oracle_rows, projection_error


def _case():
    coords = scenes.shell(16, 5.5, 2.0, 1.0, seed=3)
    nbr = O.build_neighbor_map(coords, 3)
    f = scenes.normal_features(len(coords), 24, seed=4)
    w = O.spconv_weight_to_kio(scenes.conv_weight(40, 24, 3, seed=5))
    b = np.random.default_rng(6).standard_normal(40).astype(np.float32)
    out = O.sparse_conv3d(f, nbr, w, b, accum=np.float64)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    return t(f), t(nbr), t(w), t(b), t(out)


def test_projection_accepts_the_oracle_and_rejects_one_bad_row():
    f, nbr, w, b, out = _case()
    assert projection_error(out, f, nbr, w, b) < 1e-12
    bad = out.clone()
    bad[len(bad) // 2] *= -1.0
    assert projection_error(bad, f, nbr, w, b) > 0.05


def test_projection_rejects_a_wrong_offset_weight():
    f, nbr, w, b, out = _case()
    w2 = w.clone()
    w2[4] = 0.0
    assert projection_error(out, f, nbr, w2, b) > 0.05


def test_oracle_rows_match_the_full_oracle():
    f, nbr, w, b, out = _case()
    rows = np.array([0, 7, len(out) - 1])
    got = oracle_rows(f, nbr, rows, w.numpy(), b.numpy())
    np.testing.assert_allclose(got, out.numpy()[rows], rtol=1e-5, atol=1e-5)
