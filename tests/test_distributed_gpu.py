"""Morton-range partition of one scene over two GPUs: NCCL point-to-point halo exchange plus the
tensor-core conv on each rank must reproduce the single-GPU conv of the whole scene."""

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
