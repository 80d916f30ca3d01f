"""Host-side logic of bench.py that needs no GPU: binding a rank to its GPU's local CPUs
(through a fake NVML) and giving the CPU baseline the full CPU set back afterwards, and the
batch sharding of the occupancy/width sweep over torchrun ranks."""

from __future__ import annotations

import os
import sys
import types

import numpy as np
import pytest
import torch

import bench


@pytest.fixture
def restore_affinity():
    before = os.sched_getaffinity(0)
    yield before
    os.sched_setaffinity(0, before)
    bench._HOST_CPUS = None


def _fake_nvml(local: set[int], fail: bool = False):
    nvml = types.ModuleType("pynvml")

    def handle_by_uuid(uuid):
        assert uuid == "GPU-fake-uuid"
        if fail:
            raise RuntimeError("no NVML")
        return "handle"

    def cpu_affinity(handle, words):
        out = [0] * words
        for c in local:
            out[c // 64] |= 1 << (c % 64)
        return out

    nvml.nvmlInit = lambda: None
    nvml.nvmlDeviceGetHandleByUUID = handle_by_uuid
    nvml.nvmlDeviceGetCpuAffinity = cpu_affinity
    return nvml


def _fake_props(monkeypatch):
    monkeypatch.setattr(torch.cuda, "get_device_properties",
                        lambda idx: types.SimpleNamespace(uuid="fake-uuid"))


def test_binds_to_gpu_local_cpus_and_restores(monkeypatch, restore_affinity):
    allowed = sorted(restore_affinity)
    if len(allowed) < 2:
        pytest.skip("needs two CPUs")
    extra = 64 * ((max(allowed) + 64) // 64) - 1  # within the words asked for, maybe not allowed
    local = set(allowed[: len(allowed) // 2]) | ({extra} - set(allowed))
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml(local))
    _fake_props(monkeypatch)
    bench.bind_to_gpu_cpus(0)
    assert os.sched_getaffinity(0) == set(allowed[: len(allowed) // 2])
    assert bench._HOST_CPUS == set(allowed)
    bench.use_all_host_cores()
    assert os.sched_getaffinity(0) == set(allowed)


def test_binding_is_a_no_op_without_nvml_or_when_all_cpus_are_local(monkeypatch,
                                                                     restore_affinity):
    allowed = set(restore_affinity)
    _fake_props(monkeypatch)
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml(allowed, fail=True))
    bench.bind_to_gpu_cpus(0)
    assert os.sched_getaffinity(0) == allowed and bench._HOST_CPUS is None
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml(allowed))
    bench.bind_to_gpu_cpus(0)
    assert os.sched_getaffinity(0) == allowed and bench._HOST_CPUS is None


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8, 16])
def test_sweep_batch_shards_partition_the_batch(world):
    """Every sweep element lands on exactly one rank, in order, its batch index rebased to 0 on
    that rank: the shards together are the whole batch."""

    from mlx_diffuser_b200 import scenes

    full = scenes.batched([scenes.uniform(16, 0.05, 700 + b) for b in range(bench.SWEEP_BATCH)])
    parts = [bench.batch_shard(full, bench.SWEEP_BATCH, world, r) for r in range(world)]
    assert sum(len(p) for p in parts) == len(full)
    rebuilt = []
    for r, p in enumerate(parts):
        lo = r * bench.SWEEP_BATCH // world
        hi = (r + 1) * bench.SWEEP_BATCH // world
        assert p.dtype == full.dtype and p.flags.c_contiguous
        assert set(np.unique(p[:, 0])) == set(range(hi - lo))
        q = p.copy()
        q[:, 0] += lo
        rebuilt.append(q)
    assert np.array_equal(np.concatenate(rebuilt), full)


def test_sweep_batch_shard_rejects_more_ranks_than_elements_and_parses_cells():
    full = np.zeros((4, 4), np.int32)
    with pytest.raises(ValueError):
        bench.batch_shard(full, 4, 5, 0)
    with pytest.raises(ValueError):
        bench.batch_shard(full, 4, 2, 2)
    args = types.SimpleNamespace(sweep_cells="")
    assert bench.sweep_cells(args) == bench.SWEEP_CELLS
    args.sweep_cells = "64:0.08,128:0.02"
    assert bench.sweep_cells(args) == [(64, 0.08), (128, 0.02)]
