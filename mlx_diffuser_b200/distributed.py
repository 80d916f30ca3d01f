"""Multi-GPU partitioning of the sparse-voxel path: one process per GPU.

Two modes, neither of which exists in mlx_diffuser (it runs on one Apple GPU):

* **Batch sharding** (:func:`batch_shard`): batch elements never share a neighbour -- the
  reference's neighbour key includes the batch index (``src/mlx_diffuser/layers/sparse.py:159,
  174``) -- so each rank takes whole elements and the data path needs no communication.

* **Morton-range partition of one scene** (:class:`HaloPlan`): voxels are sorted by the
  Morton code of (x, y, z) and cut into contiguous, equally sized ranges. A rank owns the
  output rows of its range; its *halo* is the set of rows owned elsewhere that are kernel
  neighbours of its own rows. Before every convolution the halo feature rows are exchanged
  with NCCL point-to-point sends/receives (``torch.distributed.batch_isend_irecv``) into a
  local buffer laid out ``[own rows; halo rows grouped by owner]``; the convolution then runs
  on the local buffer with a local neighbour map. No kernel reads another GPU's memory.

The plan is plain torch tensor logic, so it runs on CPU ``gloo`` ranks as well as on GPUs.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

# ---- batch sharding -----------------------------------------------------------------------


def batch_shard(coords: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Row indices of the batch elements assigned to ``rank``.

    Elements are dealt in contiguous blocks balanced by voxel count (greedy cut of the
    cumulative counts), so each rank keeps whole elements in their original order.
    """

    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    b = coords[:, 0].long()
    if b.numel() == 0:
        return torch.zeros(0, dtype=torch.long, device=coords.device)
    counts = torch.bincount(b - b.min())
    cum = torch.cumsum(counts, 0)
    total = int(cum[-1])
    # element e goes to the rank whose share contains the element's midpoint
    mid = cum - counts.div(2, rounding_mode="floor")
    owner = torch.clamp((mid * world) // max(total, 1), max=world - 1)
    mine = torch.nonzero(owner == rank).flatten() + b.min()
    return torch.nonzero(torch.isin(b, mine)).flatten()


# ---- Morton ranges + halo -----------------------------------------------------------------


def _spread_bits(v: torch.Tensor) -> torch.Tensor:
    """Insert two zero bits between the low 21 bits of ``v`` (int64)."""

    v = v & 0x1FFFFF
    v = (v | (v << 32)) & 0x1F00000000FFFF
    v = (v | (v << 16)) & 0x1F0000FF0000FF
    v = (v | (v << 8)) & 0x100F00F00F00F00F
    v = (v | (v << 4)) & 0x10C30C30C30C30C3
    v = (v | (v << 2)) & 0x1249249249249249
    return v


def morton_codes(coords: torch.Tensor) -> torch.Tensor:
    """63-bit Morton code of (x, y, z) relative to the scene's minimum corner."""

    xyz = coords[:, 1:].long()
    xyz = xyz - xyz.min(dim=0).values
    if xyz.numel() and int(xyz.max()) >= (1 << 21):
        raise ValueError("scene extent above 2^21 voxels per axis")
    return (_spread_bits(xyz[:, 0]) << 2) | (_spread_bits(xyz[:, 1]) << 1) | _spread_bits(xyz[:, 2])


@dataclass
class HaloPlan:
    """One rank's share of a Morton-partitioned scene.

    ``own``: global rows this rank owns (Morton order). ``halo``: global rows it reads from
    other ranks, grouped by owner. ``local_nbr``: neighbour map over the local row buffer
    ``[own; halo]`` (halo rows carry no neighbours: their outputs are never used).
    ``send_idx[s]``: local rows to send to rank ``s``; ``recv_count[s]`` / ``recv_offset[s]``:
    where rank ``s``'s rows land inside the halo block.
    """

    rank: int
    world: int
    own: torch.Tensor
    halo: torch.Tensor
    local_nbr: torch.Tensor
    send_idx: list[torch.Tensor]
    recv_count: list[int]
    recv_offset: list[int]
    schedule: tuple | None = None  # conv row schedule of local_nbr, built on first use

    @property
    def num_own(self) -> int:
        return int(self.own.numel())

    @property
    def num_local(self) -> int:
        return int(self.own.numel() + self.halo.numel())

    @staticmethod
    def build(coords: torch.Tensor, nbr: torch.Tensor, rank: int, world: int) -> HaloPlan:
        """Plan for ``rank`` from the global coordinates and global neighbour map (every rank
        computes every rank's ownership identically, so the plans agree without messages)."""

        n = coords.shape[0]
        dev = coords.device
        order = torch.argsort(morton_codes(coords), stable=True)
        bounds = [(r * n) // world for r in range(world + 1)]
        owner = torch.empty(n, dtype=torch.long, device=dev)
        for r in range(world):
            owner[order[bounds[r] : bounds[r + 1]]] = r

        def halo_of(r: int) -> torch.Tensor:
            own_r = order[bounds[r] : bounds[r + 1]]
            nb = nbr[own_r].long()
            need = torch.unique(nb[nb >= 0])
            need = need[owner[need] != r]
            # group by owner, then by global row
            key = owner[need] * n + need
            return need[torch.argsort(key)]

        own = order[bounds[rank] : bounds[rank + 1]]
        halo = halo_of(rank)
        local_of = torch.full((n,), -1, dtype=torch.long, device=dev)
        local_of[own] = torch.arange(own.numel(), device=dev)
        local_of[halo] = own.numel() + torch.arange(halo.numel(), device=dev)
        nb = nbr[own].long()
        mapped = torch.where(nb >= 0, local_of[nb.clamp(min=0)], torch.full_like(nb, -1))
        local_nbr = torch.cat(
            [mapped, torch.full((halo.numel(), nbr.shape[1]), -1, dtype=torch.long, device=dev)]
        ).to(torch.int32)

        recv_count, recv_offset = [], []
        halo_owner = owner[halo]
        off = 0
        for s in range(world):
            c = int((halo_owner == s).sum())
            recv_count.append(c)
            recv_offset.append(off)
            off += c
        send_idx = []
        for s in range(world):
            if s == rank:
                send_idx.append(torch.zeros(0, dtype=torch.long, device=dev))
                continue
            h = halo_of(s)
            rows = h[owner[h] == rank]  # sorted by global row, as rank s expects them
            send_idx.append(local_of[rows])
        return HaloPlan(rank, world, own, halo, local_nbr, send_idx, recv_count, recv_offset)

    def exchange(self, local: torch.Tensor, gather=None, group=None) -> None:
        """Fill the halo block of ``local`` ([num_local, C]) from the owning ranks.

        ``gather(src, index)`` builds each contiguous send buffer (defaults to
        ``index_select``; on GPUs the library's row-gather kernel is passed in).
        """

        if local.shape[0] != self.num_local:
            raise ValueError("local feature buffer does not match the plan")
        gather = gather or (lambda src, idx: src.index_select(0, idx))
        ops = []
        sends = []
        for s in range(self.world):
            if s == self.rank:
                continue
            if self.send_idx[s].numel():
                buf = gather(local, self.send_idx[s]).contiguous()
                sends.append(buf)
                ops.append(dist.P2POp(dist.isend, buf, s, group))
            if self.recv_count[s]:
                start = self.num_own + self.recv_offset[s]
                view = local[start : start + self.recv_count[s]]
                ops.append(dist.P2POp(dist.irecv, view, s, group))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()


# ---- GPU helpers ------------------------------------------------------------------------------


def gather_rows(src: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """``src[index]`` for a CUDA ``[rows, C]`` tensor, through the library's row-gather kernel
    (used to build the contiguous send buffers of :meth:`HaloPlan.exchange`)."""

    from . import _native as N

    src = src.contiguous()
    idx = index.to(device=src.device, dtype=torch.int32).contiguous()
    out = torch.empty((idx.numel(), src.shape[1]), dtype=src.dtype, device=src.device)
    if idx.numel() == 0 or src.shape[1] == 0:
        return out
    code = N.DTYPE_CODE.get(src.dtype)
    if code is None:
        raise ValueError(f"gather_rows: unsupported dtype {src.dtype}")
    rc = N.load().sv_upsample_features(
        src.data_ptr(), src.shape[0], src.shape[1], code, idx.data_ptr(), idx.numel(),
        out.data_ptr(), N.status_word(src.device).data_ptr(), N.stream(src.device),
    )
    N.check(rc, "gather_rows")
    return out


def halo_conv(
    plan: HaloPlan,
    local: torch.Tensor,
    weight_oki: torch.Tensor,
    bias: torch.Tensor | None,
    *,
    group=None,
) -> torch.Tensor:
    """One submanifold conv of a Morton-partitioned scene on this rank.

    ``local`` is the rank's ``[own; halo]`` feature buffer (only the own rows need to be
    filled); the halo rows are exchanged with NCCL point-to-point first, then the conv runs on
    the local buffer with the plan's local map. Returns the outputs of the rank's own rows.
    ``weight_oki`` is the spconv ``(O, k, k, k, I)`` weight in the feature dtype.
    """

    from .kernels.sparse import conv3d_forward
    from . import _native as N
    from .layers.sparse import conv_row_order

    plan.exchange(local, gather=gather_rows, group=group)
    if plan.local_nbr.device != local.device:
        plan.local_nbr = plan.local_nbr.to(local.device)
    nbr = plan.local_nbr
    if plan.schedule is None:
        plan.schedule = conv_row_order(nbr)
    row_order, tile_order = plan.schedule
    cout = weight_oki.shape[0]
    out = conv3d_forward(local.contiguous(), nbr, weight_oki.contiguous(), N.SV_WEIGHT_OKI, bias,
                         cout, row_order=row_order, tile_order=tile_order)
    return out[: plan.num_own]
