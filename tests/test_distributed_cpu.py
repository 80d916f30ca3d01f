"""Multi-rank host logic on CPU ``gloo`` ranks (world size 2 and 3): batch sharding and the
Morton-range halo plan + exchange. The local convolution in these tests is the oracle, so the
check is that partitioned results equal the single-device reference exactly."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mlx_diffuser_b200 import scenes
from mlx_diffuser_b200.distributed import HaloPlan, batch_shard, morton_codes
from oracle import sparse_oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _scene():
    coords = scenes.shell_union(40, 3, seed=5, thickness=2.5)
    feats = scenes.normal_features(len(coords), 8, seed=6)
    weight = O.spconv_weight_to_kio(scenes.conv_weight(5, 8, 3, seed=7))
    bias = np.linspace(-1, 1, 5).astype(np.float32)
    return coords, feats, weight, bias


def _halo_worker(rank: int, world: int, port: int, errors):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        coords, feats, weight, bias = _scene()
        nbr = O.build_neighbor_map(coords, 3)
        plan = HaloPlan.build(torch.from_numpy(coords), torch.from_numpy(nbr), rank, world)
        local = torch.zeros((plan.num_local, feats.shape[1]))
        local[: plan.num_own] = torch.from_numpy(feats)[plan.own]
        plan.exchange(local)
        assert torch.equal(local[plan.num_own :], torch.from_numpy(feats)[plan.halo])
        out = O.sparse_conv3d(local.numpy(), plan.local_nbr.numpy(), weight, bias)
        ref = O.sparse_conv3d(feats, nbr, weight, bias)
        np.testing.assert_array_equal(out[: plan.num_own], ref[plan.own.numpy()])
        # every row is owned exactly once across ranks
        counts = torch.tensor([plan.num_own])
        dist.all_reduce(counts)
        assert int(counts) == len(coords)
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported through the queue
        errors.put(f"rank {rank}: {e!r}")
        raise


@pytest.mark.parametrize("world", [2, 3])
def test_halo_exchange_reproduces_single_device_conv(world):
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_halo_worker, args=(r, world, port, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs)


def test_halo_is_small_for_shells():
    coords, _, _, _ = _scene()
    nbr = torch.from_numpy(O.build_neighbor_map(coords, 3))
    c = torch.from_numpy(coords)
    plans = [HaloPlan.build(c, nbr, r, 4) for r in range(4)]
    halo = sum(p.halo.numel() for p in plans)
    assert sum(p.num_own for p in plans) == len(coords)
    assert halo < 0.35 * len(coords)
    # send and receive lists agree pairwise
    for r, pr in enumerate(plans):
        for s, ps in enumerate(plans):
            if r != s:
                assert pr.send_idx[s].numel() == ps.recv_count[r]


def test_morton_codes_interleave_bits():
    c = torch.tensor([[0, 0, 0, 0], [0, 1, 0, 0], [0, 0, 1, 0], [0, 0, 0, 1], [0, 3, 3, 3]])
    assert morton_codes(c).tolist() == [0, 4, 2, 1, 63]


def test_batch_shard_keeps_whole_elements_balanced():
    coords = torch.from_numpy(scenes.batched([scenes.uniform(16, 0.1 + 0.05 * b, b) for b in range(7)]))
    for world in (1, 2, 3, 8):
        parts = [batch_shard(coords, r, world) for r in range(world)]
        allrows = torch.cat(parts).sort().values
        assert torch.equal(allrows, torch.arange(len(coords)))
        for p in parts:
            if p.numel():
                elems = coords[p, 0].unique()
                for e in elems:
                    assert int((coords[:, 0] == e).sum()) == int((coords[p, 0] == e).sum())


def test_interior_boundary_split_covers_own_rows():
    coords, _, _, _ = _scene()
    nbr = torch.from_numpy(O.build_neighbor_map(coords, 3))
    c = torch.from_numpy(coords)
    for r in range(3):
        plan = HaloPlan.build(c, nbr, r, 3)
        interior, boundary = plan.split()
        assert torch.equal(torch.sort(torch.cat([interior, boundary])).values,
                           torch.arange(plan.num_own))
        nb = plan.local_nbr
        assert not bool((nb[interior] >= plan.num_own).any())
        assert bool((nb[boundary] >= plan.num_own).any(dim=1).all())
        assert interior.numel() > boundary.numel()  # Morton ranges keep most rows interior


@pytest.mark.parametrize("world", [2, 3, 4])
def test_peer_push_lists_fill_every_halo(world):
    """Simulate the NVLink push on CPU: every rank stores its rows where push_lists says, and
    each rank's halo block then equals the rows the NCCL exchange would deliver."""

    from mlx_diffuser_b200.distributed import push_lists

    coords, feats, _, _ = _scene()
    nbr = torch.from_numpy(O.build_neighbor_map(coords, 3))
    c = torch.from_numpy(coords)
    f = torch.from_numpy(feats)
    plans = [HaloPlan.build(c, nbr, r, world) for r in range(world)]
    locals_ = []
    for p in plans:
        buf = torch.full((p.num_local, f.shape[1]), float("nan"))
        buf[: p.num_own] = f[p.own]
        locals_.append(buf)
    num_own = [p.num_own for p in plans]
    recv_off = [p.recv_offset for p in plans]
    for s, p in enumerate(plans):
        rows, dst, peers, receivers = push_lists(p, num_own, recv_off)
        for j in range(rows.numel()):
            r = receivers[int(peers[j])]
            assert plans[r].num_own <= int(dst[j]) < plans[r].num_local  # only halo rows
            locals_[r][int(dst[j])] = locals_[s][int(rows[j])]
    for p, buf in zip(plans, locals_):
        assert torch.equal(buf[p.num_own:], f[p.halo])
