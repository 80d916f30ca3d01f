"""The allocation-free kernel map, ``sv_kmap_build_static``, called through the C ABI.

Some callers of this library cannot allocate device memory: a host application that keeps
all GPU memory to itself and forbids its plugins from calling cudaMalloc, or a caller from
another language that holds only its own input and output buffers. For them the kernel map can
use a hash table compiled into the library instead of a caller-provided workspace. This test
checks that entry point against the workspace version, ``sv_kmap_build``, on calls in a row
(growing to exactly the stated maximum and shrinking again, so stale table contents from a
larger call would show, and an empty input), and that it refuses inputs above its stated
maximum. It lives in its own file, collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from mlx_diffuser_b200 import _native as N
from mlx_diffuser_b200 import scenes

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
MAX_ROWS = 524288  # SV_KMAP_STATIC_MAX_ROWS in include/sparsevox.h
INT3 = ctypes.c_int * 3


def _static_map(coords: torch.Tensor, kernel=(3, 3, 3), dilation=(1, 1, 1)) -> torch.Tensor:
    lib = N.load()
    n = coords.shape[0]
    kvol = kernel[0] * kernel[1] * kernel[2]
    nbr = torch.empty((n, kvol), dtype=torch.int32, device=DEV)
    rc = lib.sv_kmap_build_static(coords.data_ptr(), n, INT3(*kernel), INT3(*dilation),
                                  nbr.data_ptr(), N.status_word(DEV).data_ptr(), N.stream(DEV))
    N.check(rc, "sv_kmap_build_static")
    return nbr


def _workspace_map(coords: torch.Tensor, kernel=(3, 3, 3), dilation=(1, 1, 1)) -> torch.Tensor:
    lib = N.load()
    n = coords.shape[0]
    kvol = kernel[0] * kernel[1] * kernel[2]
    nbr = torch.empty((n, kvol), dtype=torch.int32, device=DEV)
    slots = lib.sv_kmap_table_slots(n)
    ws = torch.empty(lib.sv_kmap_workspace_bytes(slots), dtype=torch.uint8, device=DEV)
    rc = lib.sv_kmap_build(coords.data_ptr(), n, INT3(*kernel), INT3(*dilation), nbr.data_ptr(),
                           slots, ws.data_ptr(), ws.numel(), N.status_word(DEV).data_ptr(),
                           N.stream(DEV))
    N.check(rc, "sv_kmap_build")
    return nbr


def _full_box() -> np.ndarray:
    """Exactly MAX_ROWS distinct rows (a dense 64 x 64 x 128 box, rows shuffled): the table then
    uses every slot of the library's array, up to its last word."""

    g = np.stack(np.meshgrid(np.arange(64), np.arange(64), np.arange(128), indexing="ij"), -1)
    xyz = g.reshape(-1, 3)[np.random.default_rng(5).permutation(MAX_ROWS)]
    out = np.zeros((MAX_ROWS, 4), np.int32)
    out[:, 1:] = xyz
    return out


def test_static_kmap_matches_workspace_kmap_on_consecutive_calls():
    """Calls in a row, growing and shrinking: a small set with duplicate rows and an anisotropic
    kernel, then exactly the maximum row count (every slot of the array), then a ~237k-row scene,
    then the small set again (stale table contents from the larger calls would show), then an
    empty input. Each map must equal the workspace version's bit for bit."""

    torch.cuda.set_device(DEV)
    dup = scenes.shell(16, 5.5, 2.0, 1.0, seed=4)
    small = np.concatenate([dup, dup[::7]])  # with duplicate rows
    calls = [(small, (3, 1, 5), (2, 1, 1)), (_full_box(), (3, 3, 3), (1, 1, 1)),
             (scenes.scene128(0), (3, 3, 3), (1, 1, 1)), (small, (3, 3, 3), (1, 1, 1))]
    for coords_np, kernel, dilation in calls:
        coords = torch.from_numpy(np.ascontiguousarray(coords_np)).to(DEV)
        got = _static_map(coords, kernel, dilation)
        want = _workspace_map(coords, kernel, dilation)
        torch.cuda.synchronize()
        assert torch.equal(got, want), len(coords_np)
    empty = torch.zeros((0, 4), dtype=torch.int32, device=DEV)
    assert _static_map(empty).shape == (0, 27)
    N.check_device_status(DEV)


def test_static_kmap_rejects_inputs_above_its_maximum():
    coords = torch.zeros((MAX_ROWS + 1, 4), dtype=torch.int32, device=DEV)
    nbr = torch.empty((1, 27), dtype=torch.int32, device=DEV)
    lib = N.load()
    rc = lib.sv_kmap_build_static(coords.data_ptr(), MAX_ROWS + 1, INT3(3, 3, 3), INT3(1, 1, 1),
                                  nbr.data_ptr(), None, N.stream(DEV))
    assert rc == N.SV_ERR_UNSUPPORTED
    assert str(MAX_ROWS) in lib.sv_last_error().decode()
