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
  on the local buffer with a local neighbour map. :class:`PeerHalo` does the same exchange
  without NCCL: the owner's kernel stores the rows straight into the peers' buffers over NVLink
  (CUDA IPC mappings) and raises flags the receivers wait on, so the interior rows' convolution
  overlaps the transfer. No kernel reads another GPU's memory, and only this library's own
  kernels write it.

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
    split_schedule: tuple | None = None  # (interior rows, tiles, boundary rows, tiles)
    fused_schedule: tuple | None = None  # (rows, tiles, first halo tile) for one launch

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

        for req in self.exchange_async(local, gather, group):
            req.wait()

    def exchange_async(self, local: torch.Tensor, gather=None, group=None) -> list:
        """Start the halo exchange and return its requests without waiting. The own rows of
        ``local`` may be read meanwhile (the interior rows' convolution); the halo block is
        valid once every request has been waited on. The send buffers are kept on the plan
        until the next exchange starts."""

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
        self._inflight_sends = sends
        return dist.batch_isend_irecv(ops) if ops else []

    def split(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Own local rows whose neighbours are all own rows (``interior``: computable before the
        exchange completes) and the rest (``boundary``), as int64 local row indices."""

        nb = self.local_nbr[: self.num_own]
        needs_halo = (nb >= self.num_own).any(dim=1)
        rows = torch.arange(self.num_own, device=nb.device)
        return rows[~needs_halo], rows[needs_halo]


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


def _subset_schedule(nbr: torch.Tensor, subset: torch.Tensor):
    """Row schedule (rows in schedule order, tile order) of the rows ``subset`` of a map."""

    from .layers.sparse import conv_row_order

    if subset.numel() == 0:
        return subset.to(torch.int32), None
    order, tiles = conv_row_order(nbr[subset].contiguous())
    rows = subset[order.long()] if order is not None else subset
    return rows.to(torch.int32).contiguous(), tiles


def halo_conv_overlapped(
    plan: HaloPlan,
    local: torch.Tensor,
    weight_oki: torch.Tensor,
    bias: torch.Tensor | None,
    *,
    out: torch.Tensor | None = None,
    group=None,
) -> torch.Tensor:
    """:func:`halo_conv` with the exchange hidden behind compute: the NCCL send/receive of the
    halo rows is started, the rows whose neighbours are all own rows are convolved meanwhile
    (they read only the own block of ``local``), and the boundary rows follow once the halo
    has arrived. Returns ``out`` ([num_local, Cout]); its own rows hold the result."""

    from .kernels.sparse import conv3d_forward
    from . import _native as N

    if plan.local_nbr.device != local.device:
        plan.local_nbr = plan.local_nbr.to(local.device)
    nbr = plan.local_nbr
    if plan.split_schedule is None:
        interior, boundary = plan.split()
        plan.split_schedule = (*_subset_schedule(nbr, interior), *_subset_schedule(nbr, boundary))
    in_rows, in_tiles, bd_rows, bd_tiles = plan.split_schedule
    cout = weight_oki.shape[0]
    if out is None:
        out = torch.empty((plan.num_local, cout), dtype=local.dtype, device=local.device)
    feats = local.contiguous()
    w = weight_oki.contiguous()
    reqs = plan.exchange_async(feats, gather=gather_rows, group=group)
    conv3d_forward(feats, nbr, w, N.SV_WEIGHT_OKI, bias, cout, rows=in_rows, tile_order=in_tiles,
                   out=out)
    for req in reqs:
        req.wait()
    conv3d_forward(feats, nbr, w, N.SV_WEIGHT_OKI, bias, cout, rows=bd_rows, tile_order=bd_tiles,
                   out=out)
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


# ---- halo exchange over NVLink peer memory ---------------------------------------------------


def push_lists(plan: HaloPlan, peer_num_own: list[int], peer_recv_offset: list[list[int]]):
    """Where this rank's rows go in its peers' buffers: ``(rows, dst_rows, peers)`` over every
    peer this rank sends to, with ``dst_rows`` the row inside peer s's local buffer
    ``[own; halo by owner]`` (its own-row count plus its receive offset for this rank), and the
    list of receiving peers. Pure tensor logic, the same on every device."""

    rows, dst, peer_ids, receivers = [], [], [], []
    for s in range(plan.world):
        idx = plan.send_idx[s]
        if s == plan.rank or idx.numel() == 0:
            continue
        receivers.append(s)
        start = peer_num_own[s] + peer_recv_offset[s][plan.rank]
        rows.append(idx)
        dst.append(start + torch.arange(idx.numel(), device=idx.device))
        peer_ids.append(torch.full((idx.numel(),), len(receivers) - 1, device=idx.device))
    if not rows:
        empty = torch.zeros(0, dtype=torch.int32)
        return empty, empty, empty, receivers
    cat = lambda parts: torch.cat(parts).to(torch.int32)  # noqa: E731
    return cat(rows), cat(dst), cat(peer_ids), receivers


class PeerHalo:
    """Halo exchange of one feature buffer ``local`` ([num_local, C], CUDA) of a HaloPlan over
    NVLink peer memory (``sv_ipc_*`` / ``sv_halo_*``). Every rank builds it collectively once
    (the IPC handles travel through the process group); after that an exchange is only
    kernels on the current stream -- no collective, no host synchronisation:

    * :meth:`push` waits until the receivers have acknowledged the previous exchange, stores
      this rank's rows into their halo blocks, and raises their data flags;
    * :meth:`wait` makes the stream wait (bounded) for every sender's data flag;
    * :meth:`ack` tells the senders their rows have been consumed.
    """

    def __init__(self, plan: HaloPlan, local: torch.Tensor, group=None):
        import ctypes

        from . import _native as N

        if local.shape[0] != plan.num_local or not local.is_contiguous() or not local.is_cuda:
            raise ValueError("PeerHalo needs the plan's contiguous CUDA local buffer")
        self.plan = plan
        self.local = local
        self.row_bytes = local.shape[1] * local.element_size()
        world, rank = plan.world, plan.rank
        dev = local.device
        self.lib = N.load()
        self.status = N.status_word(dev)
        # flags[0, s]: data epoch pushed by sender s; flags[1, r]: epoch receiver r acknowledged
        self.flags = torch.zeros((2, world), dtype=torch.int64, device=dev)
        torch.cuda.synchronize(dev)

        def handle(t):
            h = (ctypes.c_char * 64)()
            off = ctypes.c_int64(0)
            N.check(self.lib.sv_ipc_handle(t.data_ptr(), h, ctypes.byref(off)), "sv_ipc_handle")
            return bytes(h), int(off.value)

        mine = {"local": handle(local), "flags": handle(self.flags), "num_own": plan.num_own,
                "num_local": plan.num_local, "recv_offset": list(plan.recv_offset)}
        infos = [None] * world
        dist.all_gather_object(infos, mine, group=group)
        self._opened: dict[bytes, int] = {}

        def open_ptr(h_off) -> int:
            h, off = h_off
            if h not in self._opened:
                base = ctypes.c_void_p(0)
                N.check(self.lib.sv_ipc_open(h, ctypes.byref(base)), "sv_ipc_open")
                self._opened[h] = int(base.value)
            return self._opened[h] + off

        rows, dst, peers, receivers = push_lists(
            plan, [i["num_own"] for i in infos], [i["recv_offset"] for i in infos])
        self.rows, self.dst, self.peers = rows.to(dev), dst.to(dev), peers.to(dev)
        self.receivers = receivers
        self.senders = [s for s in range(world) if s != rank and plan.recv_count[s] > 0]
        peer_ptrs = {s: open_ptr(infos[s]["local"]) for s in receivers}
        peer_flags = {s: open_ptr(infos[s]["flags"]) for s in set(receivers) | set(self.senders)}
        own_flags = self.flags.data_ptr()
        i64 = 8
        P = ctypes.c_void_p
        self._bases = (P * 8)(*[peer_ptrs[s] for s in receivers])
        self._peer_rows = (ctypes.c_int64 * 8)(*[infos[s]["num_local"] for s in receivers])
        # push: wait for receivers' acks (in my flags row 1), raise their data flag (row 0, me)
        self._ack_in = (P * 8)(*[own_flags + (world + s) * i64 for s in receivers])
        self._data_out = (P * 8)(*[peer_flags[s] + rank * i64 for s in receivers])
        # wait: senders' data flags in my row 0; ack: my ack in each sender's row 1
        self._data_in = (P * 8)(*[own_flags + s * i64 for s in self.senders])
        self._ack_out = (P * 8)(*[peer_flags[s] + (world + rank) * i64 for s in self.senders])
        self.epoch = 0
        dist.barrier(group=group)

    def _stream(self):
        from . import _native as N

        return N.stream(self.local.device)

    def push(self) -> None:
        from . import _native as N

        self.epoch += 1
        e, s = self.epoch, self._stream()
        nr = len(self.receivers)
        N.check(self.lib.sv_halo_wait(self._ack_in, nr, e - 1, self.status.data_ptr(), s),
                "halo ack wait")
        N.check(self.lib.sv_halo_push(self.local.data_ptr(), self.plan.num_local, self.row_bytes,
                                      self.rows.data_ptr(), self.dst.data_ptr(),
                                      self.peers.data_ptr(), self.rows.numel(), self._bases,
                                      self._peer_rows, nr, self.status.data_ptr(), s),
                "halo push")
        N.check(self.lib.sv_halo_signal(self._data_out, nr, e, s), "halo signal")

    def wait(self) -> None:
        from . import _native as N

        N.check(self.lib.sv_halo_wait(self._data_in, len(self.senders), self.epoch,
                                      self.status.data_ptr(), self._stream()), "halo data wait")

    def ack(self) -> None:
        from . import _native as N

        N.check(self.lib.sv_halo_signal(self._ack_out, len(self.senders), self.epoch,
                                        self._stream()), "halo ack")

    def close(self) -> None:
        """Unmap the peers' buffers. Call on every rank after the last exchange has completed
        everywhere (e.g. after a barrier)."""

        for base in self._opened.values():
            self.lib.sv_ipc_close(base)
        self._opened.clear()


def _fused_schedule(plan: HaloPlan):
    """One schedule for both row classes: the interior rows (padded with -1 to whole 128-row
    tiles) and then the boundary rows, with the boundary tiles' order offset past the interior
    tiles. Returns (rows, tile order, tile-order position of the first boundary tile)."""

    in_rows, in_tiles, bd_rows, bd_tiles = plan.split_schedule
    dev = in_rows.device
    n_in = (in_rows.numel() + 127) // 128
    pad = torch.full((n_in * 128 - in_rows.numel(),), -1, dtype=torch.int32, device=dev)
    rows = torch.cat([in_rows, pad, bd_rows]).contiguous()
    n_bd = (bd_rows.numel() + 127) // 128

    def tiles_of(t, count):
        return t.to(torch.int32) if t is not None else torch.arange(count, dtype=torch.int32,
                                                                    device=dev)

    tiles = torch.cat([tiles_of(in_tiles, n_in)[:n_in], tiles_of(bd_tiles, n_bd)[:n_bd] + n_in])
    return rows, tiles.contiguous(), n_in


def halo_conv_p2p(
    halo: PeerHalo,
    weight_oki: torch.Tensor,
    bias: torch.Tensor | None,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """One convolution of a Morton-partitioned scene with the halo pushed over NVLink peer
    memory: push this rank's rows to its peers, convolve the interior rows meanwhile, wait for
    the peers' rows, convolve the boundary rows, acknowledge. Returns ``out``
    ([num_local, Cout]); its own rows hold the result."""

    from .kernels.sparse import conv3d_forward, conv3d_forward_halo
    from . import _native as N

    plan, local = halo.plan, halo.local
    if plan.local_nbr.device != local.device:
        plan.local_nbr = plan.local_nbr.to(local.device)
    nbr = plan.local_nbr
    if plan.split_schedule is None:
        interior, boundary = plan.split()
        plan.split_schedule = (*_subset_schedule(nbr, interior), *_subset_schedule(nbr, boundary))
    in_rows, in_tiles, bd_rows, bd_tiles = plan.split_schedule
    cout = weight_oki.shape[0]
    cin = local.shape[1]
    if out is None:
        out = torch.empty((plan.num_local, cout), dtype=local.dtype, device=local.device)
    w = weight_oki.contiguous()
    fused = (local.dtype in (torch.float16, torch.bfloat16) and cin % 32 == 0 and cout % 32 == 0
             and nbr.shape[1] <= 27)
    halo.push()
    if fused:
        # one launch: interior tiles first; the first boundary tile waits in the kernel for the
        # peers' data flags, so the transfer overlaps the interior rows' convolution
        if plan.fused_schedule is None:
            plan.fused_schedule = _fused_schedule(plan)
        rows, tiles, halo_from = plan.fused_schedule
        conv3d_forward_halo(local, nbr, w, bias, cout, rows, tiles, halo_from, halo._data_in,
                            len(halo.senders), halo.epoch, out=out)
    else:
        conv3d_forward(local, nbr, w, N.SV_WEIGHT_OKI, bias, cout, rows=in_rows,
                       tile_order=in_tiles, out=out)
        halo.wait()
        conv3d_forward(local, nbr, w, N.SV_WEIGHT_OKI, bias, cout, rows=bd_rows,
                       tile_order=bd_tiles, out=out)
    halo.ack()
    return out
