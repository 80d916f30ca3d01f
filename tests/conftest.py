"""Shared pytest configuration: the ``gpu`` marker and fixture loading."""

from __future__ import annotations

import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


TOPOLOGY = "topology"  # subdivide / attention windows / occupancy fixture, not a conv case
RESBLOCK = "resblock"  # residual-block fixture


def golden_names() -> list[str]:
    """The conv / map / pool fixtures (one input scene each)."""

    names = (os.path.splitext(os.path.basename(p))[0]
             for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))
    return sorted(n for n in names if n not in (TOPOLOGY, RESBLOCK))


def load_golden(name: str) -> dict[str, np.ndarray]:
    with np.load(os.path.join(GOLDEN_DIR, f"{name}.npz")) as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(params=golden_names())
def golden(request):
    return request.param, load_golden(request.param)


@pytest.fixture(scope="session")
def topology_golden():
    return load_golden(TOPOLOGY)


@pytest.fixture(scope="session")
def resblock_golden():
    return load_golden(RESBLOCK)
