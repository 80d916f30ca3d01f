"""Seeded synthetic voxel scenes with the shapes of the TRELLIS sparse-voxel workloads.

No dataset is involved: every scene is generated from ``numpy.random.default_rng(seed)`` so
the CUDA path, the CPU oracle and the benchmark see identical inputs.

* :func:`shell` -- the voxels within ``thickness / 2`` of a sphere whose radius is perturbed
  by a few low-frequency angular terms (amplitude ``amplitude`` voxels). A TRELLIS structured
  latent is a surface layer of this kind (about 13.5k voxels at 64^3 for a real object).
* :func:`shell_union` -- the union of several such shells at random centres.
* :func:`uniform` -- independent uniform occupancy at a given fraction.
* :func:`shell_fraction` -- a noisy shell holding a given fraction of the grid's cells.

Coordinates are int32 rows ``(batch, x, y, z)`` in lexicographic order (the order
``np.argwhere`` gives the occupancy grid, as the reference's structure decoder does).
"""

from __future__ import annotations

import numpy as np


def _perturbed_distance(grid: int, center, radius: float, amplitude: float, rng):
    ax = np.arange(grid, dtype=np.float64)
    x, y, z = np.meshgrid(ax - center[0], ax - center[1], ax - center[2], indexing="ij")
    d = np.sqrt(x * x + y * y + z * z) + 1e-9
    theta = np.arccos(np.clip(z / d, -1.0, 1.0))
    phi = np.arctan2(y, x)
    r = np.full_like(d, radius)
    for _ in range(4):
        l_freq = rng.integers(1, 4)
        m_freq = rng.integers(1, 4)
        r += (
            amplitude
            * rng.uniform(-1.0, 1.0)
            * np.cos(l_freq * theta + rng.uniform(0.0, 2 * np.pi))
            * np.cos(m_freq * phi + rng.uniform(0.0, 2 * np.pi))
        )
    return np.abs(d - r)


def _with_batch(xyz: np.ndarray, batch: int) -> np.ndarray:
    out = np.empty((len(xyz), 4), dtype=np.int32)
    out[:, 0] = batch
    out[:, 1:] = xyz
    return out


def shell(
    grid: int,
    radius: float,
    thickness: float,
    amplitude: float,
    seed: int,
    batch: int = 0,
) -> np.ndarray:
    """One noisy sphere shell centred in a ``grid``^3 box."""

    rng = np.random.default_rng(seed)
    c = (grid - 1) / 2.0
    occ = _perturbed_distance(grid, (c, c, c), radius, amplitude, rng) < thickness / 2.0
    return _with_batch(np.argwhere(occ), batch)


def shell_union(grid: int, count: int, seed: int, thickness: float = 3.0, batch: int = 0):
    """Union of ``count`` noisy shells with random centres and radii inside the box."""

    rng = np.random.default_rng(seed)
    occ = np.zeros((grid, grid, grid), dtype=bool)
    for _ in range(count):
        radius = rng.uniform(0.16, 0.3) * grid
        center = rng.uniform(radius + 2, grid - radius - 3, size=3)
        occ |= _perturbed_distance(grid, center, radius, 0.06 * radius, rng) < thickness / 2.0
    return _with_batch(np.argwhere(occ), batch)


def uniform(grid: int, fraction: float, seed: int, batch: int = 0) -> np.ndarray:
    """Independent occupancy with probability ``fraction`` per voxel."""

    rng = np.random.default_rng(seed)
    occ = rng.random((grid, grid, grid)) < fraction
    return _with_batch(np.argwhere(occ), batch)


def shell_fraction(grid: int, fraction: float, seed: int, batch: int = 0) -> np.ndarray:
    """A noisy sphere shell holding ``round(fraction * grid^3)`` voxels: the surface-shell
    layout of the occupancy sweep.

    The radius is the one at which a 2-voxel-thick shell has the target count, capped at
    0.36 * grid (so the shell stays inside the box); the shell is then the target number of
    cells nearest the perturbed sphere (it thickens instead of growing once the radius is
    capped, e.g. about 12 voxels thick at 30% of 64^3)."""

    target = int(round(fraction * grid**3))
    rng = np.random.default_rng(seed)
    radius = min(np.sqrt(target / (8.0 * np.pi)), 0.36 * grid)
    c = (grid - 1) / 2.0
    d = _perturbed_distance(grid, (c, c, c), radius, 0.08 * radius, rng).ravel()
    if target <= 0:
        return _with_batch(np.zeros((0, 3), np.int64), batch)
    # the `target` nearest cells (ties broken by cell index), in argwhere (row-major) order
    keep = np.sort(np.argsort(d, kind="stable")[:target])
    xyz = np.stack(np.unravel_index(keep, (grid, grid, grid)), axis=1)
    return _with_batch(xyz, batch)


def batched(scenes: list[np.ndarray]) -> np.ndarray:
    """Concatenate per-element scenes, renumbering the batch column 0..B-1."""

    parts = []
    for b, s in enumerate(scenes):
        s = s.copy()
        s[:, 0] = b
        parts.append(s)
    return np.concatenate(parts, axis=0) if parts else np.zeros((0, 4), np.int32)


# ---- the workloads ---------------------------------------------------------------------------


def shell64(seed: int = 0, batch: int = 0) -> np.ndarray:
    """64^3 grid, radius-24 shell, about 20k voxels."""

    return shell(64, 24.0, 2.8, 2.0, seed, batch)


def shell32(seed: int = 0, batch: int = 0) -> np.ndarray:
    """32^3 grid, radius-12.5 shell, about 6k voxels."""

    return shell(32, 12.5, 3.05, 1.5, seed, batch)


def shell32_batch(batch: int = 4, seed: int = 0) -> np.ndarray:
    """``batch`` independent 32^3 shells (seeds ``seed .. seed+batch-1``)."""

    return batched([shell32(seed + b) for b in range(batch)])


def scene128(seed: int = 0) -> np.ndarray:
    """128^3 single scene: union of 6 noisy shells, about 250k voxels."""

    return shell_union(128, 6, seed, thickness=4.1)


def normal_features(n: int, channels: int, seed: int, std: float = 1.0) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal((n, channels)) * std).astype(np.float32)


def conv_weight(cout: int, cin: int, kernel: int, seed: int) -> np.ndarray:
    """spconv-layout ``(O, k, k, k, I)`` weight with entries N(0, 1 / (k^3 * I))."""

    std = 1.0 / np.sqrt(kernel**3 * cin)
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((cout, kernel, kernel, kernel, cin)) * std).astype(np.float32)
