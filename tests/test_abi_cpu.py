"""CPU-only checks of the C-ABI library and the host-side contract (no kernel launches)."""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from mlx_diffuser_b200 import _native as N
from mlx_diffuser_b200.kernels.sparse import sparse_conv3d
from mlx_diffuser_b200.layers.sparse import (
    SparseConv3D,
    SparseTensor,
    build_neighbor_map,
    sparse_upsample,
)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols() -> list[str]:
    names = []
    for header in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if header.endswith(".h"):
            text = open(os.path.join(ROOT, "include", header)).read()
            names += re.findall(r"SV_API\s+[\w\s\*]+?\b(sv_\w+)\s*\(", text)
    return names


def test_library_exports_every_declared_symbol():
    lib = N.load()
    declared = _declared_symbols()
    assert len(declared) >= 14
    for name in declared:
        assert hasattr(lib, name), name
    # and the Python binding declares a signature for every one of them
    assert set(declared) <= set(N.EXPORTED)


def test_abi_version_and_sizes():
    lib = N.load()
    assert lib.sv_abi_version() == 1
    assert lib.sv_kmap_table_slots(0) == 64
    assert lib.sv_kmap_table_slots(1000) == 2048
    assert lib.sv_kmap_workspace_bytes(2048) == 2048 * 48
    assert lib.sv_conv_plan_workspace_bytes(0) == 0
    assert lib.sv_downsample_workspace_bytes(10) >= 10 * 28
    # KIO weight on a tensor-core shape needs a repack workspace; OKI needs none
    kio = lib.sv_conv3d_workspace_bytes(100, 64, 64, 27, 2, N.SV_WEIGHT_KIO, N.SV_CONV_AUTO)
    assert kio >= 27 * 64 * 64 * 2
    # the tensor-core path always needs its scheduler word; the CUDA-core path nothing
    assert lib.sv_conv3d_workspace_bytes(100, 64, 64, 27, 2, N.SV_WEIGHT_OKI, N.SV_CONV_AUTO) == 256
    assert lib.sv_conv3d_workspace_bytes(100, 64, 64, 27, 2, N.SV_WEIGHT_OKI, N.SV_CONV_SIMT) == 0
    # fp32 runs on the 3xTF32 kernel: scheduler word, repacked weight, its hi / lo halves
    w32 = 27 * 64 * 64 * 4
    assert lib.sv_conv3d_workspace_bytes(100, 64, 64, 27, 0, N.SV_WEIGHT_KIO,
                                         N.SV_CONV_AUTO) == 256 + 3 * w32
    assert lib.sv_conv3d_workspace_bytes(100, 64, 64, 27, 0, N.SV_WEIGHT_KIO, N.SV_CONV_SIMT) == 0
    # 8 input channels run on the tensor cores too (offsets packed four per stage)
    assert lib.sv_conv3d_workspace_bytes(100, 8, 64, 27, 2, N.SV_WEIGHT_KIO,
                                         N.SV_CONV_AUTO) == 256 + 27 * 8 * 64 * 2
    # 24 input channels: the CUDA-core kernel, no workspace
    assert lib.sv_conv3d_workspace_bytes(100, 24, 64, 27, 2, N.SV_WEIGHT_KIO, N.SV_CONV_AUTO) == 0


def test_argument_errors_are_reported_before_any_launch():
    lib = N.load()
    k = (ctypes.c_int * 3)(4, 3, 3)
    d = (ctypes.c_int * 3)(1, 1, 1)
    rc = lib.sv_kmap_build(None, 10, k, d, None, 64, None, 0, None, None)
    assert rc == N.SV_ERR_BAD_SHAPE
    assert "odd" in lib.sv_last_error().decode()
    rc = lib.sv_conv3d_forward(None, 5, 8, None, 27, None, None, None, 0, None, 8, 7, None, 0, None, 0,
                               None, None)
    assert rc == N.SV_ERR_BAD_DTYPE
    rc = lib.sv_conv3d_forward(None, 5, 8, None, 27, None, None, None, 0, None, 8, 2, None, 9, None, 0,
                               None, None)
    assert rc == N.SV_ERR_INVALID_ARGUMENT
    # nothing to do -> OK without touching the device
    assert lib.sv_conv3d_forward(None, 0, 8, None, 27, None, None, None, 0, None, 8, 2, None, 0, None, 0,
                                 None, None) == N.SV_OK
    m = ctypes.c_int64(-1)
    assert lib.sv_downsample_coords(None, 0, 2, None, None, None, None, ctypes.byref(m), None, 0,
                                    None) == N.SV_OK
    assert m.value == 0
    assert lib.sv_downsample_coords(None, 5, 0, None, None, None, None, ctypes.byref(m), None, 0,
                                    None) == N.SV_ERR_INVALID_ARGUMENT
    # topology entry points: empty inputs succeed without touching the device, bad ones fail
    shape = (ctypes.c_int64 * 4)(2, 0, 64, 64)
    strides = (ctypes.c_int64 * 4)(0, 4096, 64, 1)
    assert lib.sv_occupancy_workspace_bytes(shape) == 256
    assert lib.sv_occupancy_workspace_bytes((ctypes.c_int64 * 4)(2, 64, 64, 64)) >= 2 * 512 * 4
    assert lib.sv_occupancy_count(None, 0, shape, strides, 0.0, ctypes.byref(m), None, 0,
                                  None) == N.SV_OK
    assert m.value == 0
    assert lib.sv_occupancy_count(None, 9, shape, strides, 0.0, ctypes.byref(m), None, 0,
                                  None) == N.SV_ERR_BAD_DTYPE
    neg = (ctypes.c_int64 * 4)(2, -1, 4, 4)
    assert lib.sv_occupancy_count(None, 0, neg, strides, 0.0, ctypes.byref(m), None, 0,
                                  None) == N.SV_ERR_INVALID_ARGUMENT
    assert lib.sv_subdivide(None, 0, None, 0, None, None, None) == N.SV_OK
    assert lib.sv_subdivide(None, -1, None, 0, None, None, None) == N.SV_ERR_INVALID_ARGUMENT
    shift = (ctypes.c_int * 3)(0, 0, 0)
    assert lib.sv_window_groups(None, 0, 8, shift, None, None, ctypes.byref(m), None, 0,
                                None) == N.SV_OK
    assert lib.sv_window_groups(None, 5, -2, shift, None, None, ctypes.byref(m), None, 0,
                                None) == N.SV_ERR_INVALID_ARGUMENT
    assert lib.sv_window_groups_workspace_bytes(100) > lib.sv_downsample_workspace_bytes(100)
    with pytest.raises(ValueError):
        N.check(N.SV_ERR_BAD_SHAPE, "x")
    with pytest.raises(RuntimeError):
        N.check(N.SV_ERR_CUDA, "x")


def test_sparse_tensor_host_semantics():
    coords = torch.tensor([[0, 0, 0, 0], [1, 2, 3, 1], [1, 0, 5, 2]], dtype=torch.int64)
    feats = torch.arange(6, dtype=torch.float32).reshape(3, 2)
    t = SparseTensor(feats, coords)
    assert t.coords.dtype == torch.int32
    assert t.batch_size == 2 and t.spatial_shape == (3, 6, 3)
    assert t.shape == (2, 2) and t.num_points == 3 and t.feats is t.features
    u = t.replace(feats * 2)
    assert u.cache is t.cache and u.spatial_shape == t.spatial_shape
    assert torch.equal((t + t).features, feats * 2)
    assert torch.equal((t * torch.tensor([[1.0, 1.0], [2.0, 2.0]])).features[1], feats[1] * 2)
    assert torch.equal((1 - t).features, 1 - feats)
    assert [s.stop - s.start for s in t.batch_layout()] == [1, 2]
    d = t.dense()
    assert d.shape == (2, 3, 6, 3, 2) and torch.equal(d[1, 2, 3, 1], feats[1])
    empty = SparseTensor(torch.zeros((0, 4)), torch.zeros((0, 4), dtype=torch.int32))
    assert empty.batch_size == 0 and empty.spatial_shape == (0, 0, 0)


def test_sparse_tensor_validation_matches_reference_messages():
    with pytest.raises(ValueError, match="features must have shape"):
        SparseTensor(torch.zeros(3), torch.zeros((3, 4), dtype=torch.int32))
    with pytest.raises(ValueError, match=r"coords must have shape \(N, 4\)"):
        SparseTensor(torch.zeros((3, 2)), torch.zeros((3, 3), dtype=torch.int32))
    with pytest.raises(ValueError, match="same number of points"):
        SparseTensor(torch.zeros((2, 2)), torch.zeros((3, 4), dtype=torch.int32))
    with pytest.raises(ValueError, match="must be paired"):
        sparse_upsample(SparseTensor(torch.zeros((1, 2)), torch.zeros((1, 4), dtype=torch.int32)))
    with pytest.raises(ValueError, match="odd kernel_size"):
        SparseConv3D(2, 2, 4)
    with pytest.raises(ValueError, match="three odd dimensions"):
        build_neighbor_map(torch.zeros((1, 4), dtype=torch.int32), 2)


def test_conv_validation_matches_reference_messages():
    f = torch.zeros((4, 3))
    nbr = torch.zeros((4, 27), dtype=torch.int32)
    w = torch.zeros((27, 3, 2))
    b = torch.zeros(2)
    with pytest.raises(ValueError, match="features must be 2D"):
        sparse_conv3d(torch.zeros(4), nbr, w, b)
    with pytest.raises(ValueError, match="neighbors must have shape"):
        sparse_conv3d(f, nbr[:3], w, b)
    with pytest.raises(ValueError, match="weights must have shape"):
        sparse_conv3d(f, nbr, torch.zeros((27, 4, 2)), b)
    with pytest.raises(ValueError, match="bias must have shape"):
        sparse_conv3d(f, nbr, w, torch.zeros(3))


def test_no_cpu_fallback():
    """Valid inputs on the CPU raise instead of silently computing on the host."""

    coords = torch.zeros((2, 4), dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        build_neighbor_map(coords, 3)
    with pytest.raises(RuntimeError, match="CUDA"):
        sparse_conv3d(torch.zeros((2, 3)), torch.zeros((2, 27), dtype=torch.int32),
                      torch.zeros((27, 3, 2)), torch.zeros(2))
    conv = SparseConv3D(3, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        conv(SparseTensor(torch.zeros((2, 3)), coords))


def test_module_parameters_follow_spconv_layout():
    conv = SparseConv3D(5, 7, 3, bias=True)
    assert tuple(conv.conv.weight.shape) == (7, 3, 3, 3, 5)
    bound = 1.0 / np.sqrt(5 * 27)
    assert float(conv.conv.weight.abs().max()) <= bound
    assert torch.count_nonzero(conv.conv.bias) == 0
    conv.conv.weight = torch.zeros_like(conv.conv.weight)  # plain tensor assignment works
    nob = SparseConv3D(5, 7, 3, bias=False)
    assert not hasattr(nob.conv, "bias") and hasattr(nob.conv, "_bias")
    conv.cast_dtype(torch.float16)
    assert conv.conv.weight.dtype == torch.float16 and conv.conv.bias.dtype == torch.float16
