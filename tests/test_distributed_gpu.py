"""Morton-range partition of one scene.

* On one GPU: every rank's share of a partitioned scene (2, 4 and 8 ranks) is convolved in turn
  on the local buffer the halo exchange produces -- by the local tensor-core conv and by the
  single-launch halo conv whose in-kernel wait finds its flags already raised -- and the union of
  the ranks' own rows is compared with the fp32 oracle of the whole scene.
* On two GPUs: NCCL point-to-point and NVLink peer-memory exchanges plus the tensor-core conv on
  each rank must reproduce the single-GPU conv of the whole scene, and the fp32 oracle."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, errors):
    try:
        import torch.distributed as dist
        from datetime import timedelta

        from mlx_diffuser_b200 import scenes
        from mlx_diffuser_b200.distributed import (
            HaloPlan,
            PeerHalo,
            halo_conv,
            halo_conv_overlapped,
            halo_conv_p2p,
        )
        from mlx_diffuser_b200.kernels.sparse import conv3d_forward
        from mlx_diffuser_b200 import _native as N
        from mlx_diffuser_b200.layers.sparse import build_neighbor_map, conv_row_order

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=60))
        coords_np = scenes.shell_union(64, 4, seed=9, thickness=3.0)
        coords = torch.from_numpy(coords_np).to(dev)
        feats = torch.from_numpy(scenes.normal_features(len(coords_np), 64, 10)).to(dev, torch.bfloat16)
        w = torch.from_numpy(scenes.conv_weight(64, 64, 3, 11)).to(dev, torch.bfloat16).contiguous()
        b = torch.linspace(-1, 1, 64, device=dev).to(torch.bfloat16)
        nbr = build_neighbor_map(coords, 3)
        plan = HaloPlan.build(coords, nbr, rank, world)
        local = torch.zeros((plan.num_local, 64), device=dev, dtype=torch.bfloat16)
        local[: plan.num_own] = feats[plan.own]
        out_own = halo_conv(plan, local, w, b)
        assert torch.equal(local[plan.num_own:], feats[plan.halo])
        order, tiles = conv_row_order(nbr)
        full = conv3d_forward(feats, nbr, w, N.SV_WEIGHT_OKI, b, 64, row_order=order,
                              tile_order=tiles)
        ref = full[plan.own]
        err = (out_own.float() - ref.float()).abs().max() / ref.float().abs().max()
        assert float(err) <= 1e-6, float(err)
        # and the fp32 oracle on this rank's rows
        from oracle import sparse_oracle as O

        own_np = plan.own.cpu().numpy()
        f32 = feats.float().cpu().numpy()
        oracle = O.sparse_conv3d(f32, nbr.cpu().numpy(), O.spconv_weight_to_kio(
            w.float().cpu().numpy()), b.float().cpu().numpy())[own_np]
        got = out_own.float().cpu().numpy()
        assert float(np.abs(got - oracle).max() / np.abs(oracle).max()) <= 1e-2
        # the overlapped variant: interior rows while the exchange is in flight, then boundary
        local2 = torch.zeros_like(local)
        local2[: plan.num_own] = feats[plan.own]
        out2 = halo_conv_overlapped(plan, local2, w, b)
        assert torch.equal(local2[plan.num_own:], feats[plan.halo])
        assert torch.equal(out2[: plan.num_own], out_own)
        # NVLink peer-memory push: three exchanges in a row exercise the data / ack epochs
        local3 = torch.zeros_like(local)
        local3[: plan.num_own] = feats[plan.own]
        halo = PeerHalo(plan, local3)
        for _ in range(3):
            out3 = halo_conv_p2p(halo, w, b)
            torch.cuda.synchronize(dev)
            assert torch.equal(local3[plan.num_own:], feats[plan.halo])
            assert torch.equal(out3[: plan.num_own], out_own)
        N.check_device_status(dev)
        dist.barrier(device_ids=[rank])
        halo.close()
        N.check_device_status(dev)
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported through the queue
        errors.put(f"rank {rank}: {e!r}")
        raise


@pytest.mark.parametrize("world", [2, 4, 8])
def test_partitioned_scene_on_one_gpu_matches_oracle(world):
    """Each rank of a ``world``-way Morton partition, run one after another on one GPU: the local
    buffer is filled as the exchange would fill it (own rows, then the halo rows by owner), then
    convolved by the local tcgen05 conv and by the single-launch halo conv (its flags raised
    beforehand, so the in-kernel wait passes at once). The ranks' own rows together must equal
    the fp32 oracle of the whole scene (max relative error 1e-2) and each other (bit-exact)."""

    import ctypes

    from mlx_diffuser_b200 import _native as N
    from mlx_diffuser_b200 import scenes
    from mlx_diffuser_b200.distributed import HaloPlan, _fused_schedule, _subset_schedule
    from mlx_diffuser_b200.kernels.sparse import conv3d_forward, conv3d_forward_halo
    from mlx_diffuser_b200.layers.sparse import build_neighbor_map, conv_row_order
    from oracle import sparse_oracle as O

    dev = torch.device("cuda", 0)
    dt = torch.bfloat16
    coords_np = scenes.shell_union(64, 4, seed=9, thickness=3.0)
    n = len(coords_np)
    coords = torch.from_numpy(coords_np).to(dev)
    f_np = torch.from_numpy(scenes.normal_features(n, 64, 10)).to(dt).float().numpy()
    w_np = torch.from_numpy(scenes.conv_weight(32, 64, 3, 11)).to(dt).float().numpy()
    b_np = torch.linspace(-1, 1, 32).to(dt).float().numpy()
    feats = torch.from_numpy(f_np).to(dev, dt)
    w = torch.from_numpy(w_np).to(dev, dt).contiguous()
    b = torch.from_numpy(b_np).to(dev, dt)
    nbr = build_neighbor_map(coords, 3)
    oracle = O.sparse_conv3d(f_np, nbr.cpu().numpy(), O.spconv_weight_to_kio(w_np), b_np)
    got = torch.full((n, 32), float("nan"), device=dev)
    flags = torch.full((8,), 1 << 40, dtype=torch.int64, device=dev)  # every flag already raised
    flag_ptrs = (ctypes.c_void_p * 8)(*[flags.data_ptr() + 8 * i for i in range(8)])
    halo_total = 0
    for rank in range(world):
        plan = HaloPlan.build(coords, nbr, rank, world)
        halo_total += plan.halo.numel()
        local = torch.cat([feats[plan.own], feats[plan.halo]]).contiguous()
        lnbr = plan.local_nbr.to(dev)
        order, tiles = conv_row_order(lnbr)
        plain = conv3d_forward(local, lnbr, w, N.SV_WEIGHT_OKI, b, 32, row_order=order,
                               tile_order=tiles)
        plan.local_nbr = lnbr
        interior, boundary = plan.split()
        plan.split_schedule = (*_subset_schedule(lnbr, interior), *_subset_schedule(lnbr, boundary))
        rows, tile_list, halo_from = _fused_schedule(plan)
        fused = torch.empty((plan.num_local, 32), device=dev, dtype=dt)
        senders = sum(1 for s in range(world) if s != rank and plan.recv_count[s] > 0)
        conv3d_forward_halo(local, lnbr, w, b, 32, rows, tile_list, halo_from, flag_ptrs,
                            min(senders, 8), 1, out=fused)
        N.check_device_status(dev)
        assert torch.equal(fused[: plan.num_own], plain[: plan.num_own])
        got[plan.own] = plain[: plan.num_own].float()
    assert halo_total > 0
    assert not torch.isnan(got).any(), "a row is owned by no rank"
    err = np.abs(got.cpu().numpy() - oracle).max() / np.abs(oracle).max()
    assert err <= 1e-2, err


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_halo_conv_over_two_gpus_matches_single_gpu():
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, errors)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs)
