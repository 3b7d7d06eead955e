"""Morton-range sharding of one sparse-voxel set across ranks, with a one-voxel halo.

Large grids (the 512^3 and 1024^3 configurations) are split across the GPUs of
one box by contiguous ranges of a global Morton order: each rank owns the
voxels whose Morton code falls in its range and computes their outputs.  A
3x3x3 submanifold conv also reads neighbours owned by other ranks, so before
each conv every rank receives the features of those neighbours (its halo).

* Range boundaries are multiples of 8 in Morton code, so every 2x2x2 sibling
  group lives on one rank and stride-2 down/up convs need no exchange.
* Send lists need no existence query: rank r sends owned voxel v to rank s
  when one of v's 26 neighbour *positions* falls in s's range.  Submanifold
  neighbourhood is symmetric, so this covers every input s needs (plus a few
  voxels s never reads).
* The plan (send lists, split sizes, halo coords) is built once per coord set
  and reused by every conv layer on those coords, like the neighbour map.
* The plan orders a rank's owned rows interior first: rows none of whose 26
  neighbour positions lies in another rank's range read no halo row, so their
  outputs can be computed while the halo is in flight; boundary rows follow.
* Per layer the exchange is one ``all_to_all_single`` (NCCL on GPUs, gloo on
  CPU ranks) of the packed send rows into the halo rows of the local feature
  buffer: owned rows first (in plan order), then halo rows grouped by source
  rank.

The plan logic is device-agnostic torch code, so the same functions run on CPU
ranks (gloo) in the tests and on GPUs (NCCL) in the benchmark.
"""
from __future__ import annotations

import dataclasses

import torch

__all__ = ["morton_codes", "MortonPartition", "HaloPlan", "build_halo_plan", "exchange_halo", "local_coords",
           "owned_local", "peer_destinations", "PeerHaloExchange", "lpt_assign", "batch_rows"]

_OFFS26 = [(dx, dy, dz) for dx in (-1, 0, 1) for dy in (-1, 0, 1) for dz in (-1, 0, 1) if (dx, dy, dz) != (0, 0, 0)]


def _part1by2(v):
    v = v & 0xFFFF
    v = (v | (v << 32)) & 0x1F00000000FFFF
    v = (v | (v << 16)) & 0x1F0000FF0000FF
    v = (v | (v << 8)) & 0x100F00F00F00F00F
    v = (v | (v << 4)) & 0x10C30C30C30C30C3
    v = (v | (v << 2)) & 0x1249249249249249
    return v


def morton_codes(coords):
    """int64 code = batch (15 bits) above the 48-bit Morton interleave of (x, y, z)."""
    c = coords.to(torch.int64)
    return (c[:, 0] << 48) | (_part1by2(c[:, 1]) << 2) | (_part1by2(c[:, 2]) << 1) | _part1by2(c[:, 3])


@dataclasses.dataclass
class MortonPartition:
    """Contiguous Morton ranges, one per rank: rank s owns codes in [bounds[s], bounds[s+1])."""
    bounds: torch.Tensor  # int64 [world + 1]

    @staticmethod
    def balanced(coords, world, align=8):
        """Equal-count split of the sorted codes, each boundary rounded down to a multiple of `align`."""
        codes, _ = torch.sort(morton_codes(coords))
        n = codes.numel()
        b = [torch.iinfo(torch.int64).min]
        for s in range(1, world):
            k = min(n - 1, (s * n) // world) if n else 0
            cut = (int(codes[k]) // align) * align if n else 0
            b.append(max(cut, b[-1]))
        b.append(torch.iinfo(torch.int64).max)
        return MortonPartition(torch.tensor(b, dtype=torch.int64, device=coords.device))

    def owner(self, codes):
        return torch.searchsorted(self.bounds, codes, right=True) - 1

    def coarsen(self):
        """The same ranges one level down (codes of parents ``(b, x>>1, y>>1, z>>1)``).

        A parent's code is its children's code shifted right by 3 (the batch
        field shifts with them, so it is re-aligned).  With boundaries that
        are multiples of 8, every 2x2x2 sibling group is owned by one rank, so
        every parent is owned by the rank that owns its children and the
        stride-2 down / up convs need no exchange.
        """
        lo, hi = torch.iinfo(torch.int64).min, torch.iinfo(torch.int64).max
        out = []
        for v in self.bounds.tolist():
            if v in (lo, hi):
                out.append(v)
                continue
            b, m = v >> 48, v & ((1 << 48) - 1)
            out.append((b << 48) | (m >> 3))
        return MortonPartition(torch.tensor(out, dtype=torch.int64, device=self.bounds.device))

    def owned_rows(self, coords, rank):
        """Rows of a (global) coord array owned by `rank`, in input order."""
        return torch.nonzero(self.owner(morton_codes(coords)) == rank).squeeze(1)


@dataclasses.dataclass
class HaloPlan:
    rank: int
    world: int
    n_own: int
    n_interior: int             # local rows [0, n_interior) read no halo row
    order: torch.Tensor         # local owned row k is the caller's owned row order[k]
    send_idx: torch.Tensor      # local owned rows to pack, grouped by destination rank
    send_splits: list           # rows sent to each rank
    recv_splits: list           # rows received from each rank
    halo_coords: torch.Tensor   # (n_halo, 4) int32, grouped by source rank

    @property
    def n_halo(self):
        return int(self.halo_coords.shape[0])


def build_halo_plan(owned_coords, partition, rank, world, group=None, interior_first=True):
    """Collective: every rank calls it with its owned coords (int32 (n, 4)).

    With ``interior_first`` (default) the local order puts rows that read no
    halo row first (for convs that overlap the exchange); without it the
    local order is the caller's order (``order`` is the identity), so a
    tensor over the owned rows can be used as the local rows directly."""
    import torch.distributed as dist
    dev = owned_coords.device
    c = owned_coords.to(torch.int64)
    n = c.shape[0]
    need = torch.zeros((world, n), dtype=torch.bool, device=dev)
    for dx, dy, dz in _OFFS26:
        p = torch.stack([c[:, 0], c[:, 1] + dx, c[:, 2] + dy, c[:, 3] + dz], 1)
        ok = (p[:, 1:] >= 0).all(1) & (p[:, 1:] <= 65535).all(1)
        own = partition.owner(morton_codes(p.clamp(min=0)))
        own = torch.where(ok, own, torch.full_like(own, rank))
        need[own, torch.arange(n, device=dev)] = True
    need[rank] = False
    boundary = need.any(0)
    if interior_first:
        order = torch.cat([torch.nonzero(~boundary).squeeze(1), torch.nonzero(boundary).squeeze(1)])
        n_interior = int(n - int(boundary.sum()))
    else:
        order = torch.arange(n, device=dev)
        n_interior = 0
    local_of = torch.empty_like(order)
    local_of[order] = torch.arange(n, device=dev)
    idx, splits = [], []
    for s in range(world):
        rows = local_of[torch.nonzero(need[s]).squeeze(1)]
        idx.append(rows)
        splits.append(int(rows.numel()))
    send_idx = torch.cat(idx) if idx else torch.zeros(0, dtype=torch.int64, device=dev)
    sc = torch.tensor(splits, dtype=torch.int64, device=dev)
    rc = torch.empty_like(sc)
    dist.all_to_all_single(rc, sc, group=group)
    recv_splits = [int(v) for v in rc.tolist()]
    halo = torch.empty((sum(recv_splits), 4), dtype=owned_coords.dtype, device=dev)
    local = owned_coords.index_select(0, order)
    dist.all_to_all_single(halo, local.index_select(0, send_idx).contiguous(), recv_splits, splits, group=group)
    return HaloPlan(rank, world, n, n_interior, order, send_idx, splits, recv_splits, halo)


def owned_local(plan, t):
    """Rows of a tensor over the caller's owned rows, in the plan's local order."""
    return t.index_select(0, plan.order)


def local_coords(plan, owned_coords):
    """Coords of the local input rows: owned rows (plan order), then halo rows."""
    return torch.cat([owned_local(plan, owned_coords), plan.halo_coords], 0).contiguous()


def exchange_halo(plan, owned_feats, out=None, group=None, async_op=False):
    """Collective: returns (n_own + n_halo, C) features, owned rows first then halo rows.

    ``owned_feats`` holds the owned rows in plan order.  ``out``, when given,
    must already hold them in its first n_own rows (e.g. the previous layer
    wrote them there); only the halo rows are filled.  With ``async_op`` the
    call returns ``(out, work)`` as soon as the exchange is enqueued (NCCL runs
    it beside work queued later on the current stream) and ``work.wait()``
    orders the current stream after it.
    """
    import torch.distributed as dist
    c = owned_feats.shape[1]
    if out is None:
        out = torch.empty((plan.n_own + plan.n_halo, c), dtype=owned_feats.dtype, device=owned_feats.device)
        out[:plan.n_own].copy_(owned_feats)
    send = owned_feats.index_select(0, plan.send_idx).contiguous()
    work = dist.all_to_all_single(out[plan.n_own:], send, plan.recv_splits, plan.send_splits, group=group,
                                  async_op=async_op)
    return (out, work) if async_op else out


def peer_destinations(plan, peer_info):
    """Destination (peer, local row) of each of this rank's send rows, in send order.

    ``peer_info[s] = (n_own_s, recv_splits_s)`` of every rank s.  Rank s keeps
    its halo rows grouped by source rank after its owned rows, so row j of the
    rows this rank sends to s lands at ``n_own_s + sum(recv_splits_s[:rank]) + j``.
    Raises when the plans disagree on the row counts.
    """
    dst_peer, dst_row = [], []
    for s in range(plan.world):
        cnt = plan.send_splits[s]
        if cnt == 0:
            continue
        n_own_s, recv_s = peer_info[s]
        if recv_s[plan.rank] != cnt:
            raise RuntimeError(f"halo plan mismatch: rank {s} expects {recv_s[plan.rank]} rows from "
                               f"{plan.rank}, got {cnt}")
        first = n_own_s + sum(recv_s[:plan.rank])
        dst_peer += [s] * cnt
        dst_row += list(range(first, first + cnt))
    return dst_peer, dst_row


class _DeviceArray:
    """A raw device buffer seen as a torch tensor (``__cuda_array_interface__``)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


_TYPESTR = {torch.bfloat16: "<i2", torch.float16: "<f2", torch.float32: "<f4"}  # bf16 viewed from int16


class PeerHaloExchange:
    """Halo exchange over peer memory: one push kernel per layer, waited for by a wait kernel or by the conv.

    Every rank allocates one peer buffer (``sc_peer_alloc``) holding two local
    feature regions (owned rows then halo rows, used in alternate exchanges)
    and one flag word per source rank, and opens the other ranks' buffers by
    CUDA IPC.  ``exchange()`` stores this rank's send rows straight into the
    other ranks' halo rows of the next region and waits until every other
    rank has filled this rank's halo (``sc_halo_push`` / ``sc_halo_wait``, on
    the current stream).  ``push()`` only stores and signals; the conv that
    follows then waits inside its kernel, before its first tile that reads a
    halo row (``conv3d(..., halo_wait=...)``, e.g. on a map from
    ``concat_kmaps`` of the interior and boundary outputs).  On the 1024^3
    workload that conv ran slower inside the multi-GPU step than
    ``exchange()`` followed by a plain conv (8 GPUs: 0.243 vs 0.213 ms per
    layer), so ``exchange()`` is the faster path today.
    The caller keeps the owned rows of the region it exchanges in place
    (``region(parity)[:n_own]``); both regions start with the owned features
    given to the constructor.  Collective: all ranks build it together and
    call ``exchange()`` / ``push()`` the same number of times.
    """

    def __init__(self, plan, owned_feats, engine, group=None):
        import ctypes
        import torch.distributed as dist
        from . import _lib as L
        self.plan, self.engine, self.lib = plan, engine, engine.lib
        world, rank = plan.world, plan.rank
        dev = owned_feats.device
        dtype, channels = owned_feats.dtype, int(owned_feats.shape[1])
        self.dtype, self.channels = dtype, channels
        self.row_bytes = channels * owned_feats.element_size()
        if self.row_bytes % 16:
            raise ValueError("peer halo exchange needs rows of a multiple of 16 bytes")
        self.n_rows = plan.n_own + plan.n_halo
        self.region = (self.n_rows * self.row_bytes + 255) // 256 * 256
        total = 2 * self.region + 256
        ptr, handle = ctypes.c_void_p(), (ctypes.c_char * L.SC_IPC_HANDLE_BYTES)()
        engine.check(self.lib.sc_peer_alloc(engine.handle, total, ctypes.byref(ptr), handle), "sc_peer_alloc")
        self.base = ptr.value
        infos = [None] * world
        dist.all_gather_object(infos, (bytes(handle), plan.n_own, list(plan.recv_splits), self.region), group=group)
        self.peers = {}
        for r in range(world):
            if r == rank:
                continue
            pp = ctypes.c_void_p()
            engine.check(self.lib.sc_peer_open(engine.handle, infos[r][0], ctypes.byref(pp)), "sc_peer_open")
            self.peers[r] = pp.value
        bases = [self.base if r == rank else self.peers[r] for r in range(world)]
        dst_peer, dst_row = peer_destinations(plan, [(i[1], i[2]) for i in infos])
        rows = torch.tensor(dst_row, dtype=torch.int64)
        self.dst_off = [(rows * self.row_bytes + p * torch.tensor([infos[s][3] for s in dst_peer], dtype=torch.int64)
                         if dst_peer else rows).to(dev) for p in (0, 1)]
        self.dst_peer = torch.tensor(dst_peer, dtype=torch.int32, device=dev)
        self.src_row = plan.send_idx.to(device=dev, dtype=torch.int32).contiguous()
        self.peer_bufs = torch.tensor(bases, dtype=torch.int64, device=dev)
        self.peer_flags = torch.tensor([b + 2 * infos[r][3] for r, b in enumerate(bases)], dtype=torch.int64,
                                       device=dev)
        self.flags = self.base + 2 * self.region
        self.epoch = 0
        self.group = group
        for p in (0, 1):
            self.region_view(p)[:plan.n_own].copy_(owned_feats)
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    def next_owned_rows(self):
        """Owned rows (n_own, C) of the region the next ``exchange()`` / ``push()``
        sends from: a layer that produces this rank's features writes them
        here, and the exchange then fills the same region's halo rows."""
        return self.region_view((self.epoch + 1) & 1)[:self.plan.n_own]

    def region_view(self, parity):
        """Local features of region `parity`: (n_own + n_halo, C), owned rows first."""
        arr = _DeviceArray(self.base + parity * self.region, (self.n_rows, self.channels), _TYPESTR[self.dtype])
        t = torch.as_tensor(arr, device=torch.device("cuda", self.engine.device.index))
        return t.view(self.dtype) if self.dtype == torch.bfloat16 else t

    def exchange(self):
        """Fills the halo rows of the next region; returns that region (on the current stream)."""
        import ctypes
        local, hw = self.push()
        eng = self.engine
        eng.check(self.lib.sc_halo_wait(eng.handle, ctypes.c_void_p(hw.flags), hw.world, hw.rank, hw.epoch),
                  "sc_halo_wait")
        return local

    def push(self):
        """Starts the next exchange without waiting for it, on the current
        stream: returns the region and a :class:`HaloWait` for
        ``conv3d(..., halo_wait=...)``, which waits on the device before
        gathering halo rows.  Pair every ``push()`` with one such conv (or
        ``sc_halo_wait``) before the next ``push()``: that wait keeps this rank
        at most one exchange ahead of its peers.

        The push kernel must complete before the conv that waits for the
        peers' pushes starts (stream order): a push enqueued beside that conv
        (another stream) may find no free SM while the conv's CTAs wait for a
        peer whose own conv waits for this push, and the waits then run out."""
        from .sparse_conv import HaloWait
        self.epoch += 1
        parity = self.epoch & 1
        local = self.region_view(parity)
        self._enqueue_push(local, parity)
        p = self.plan
        return local, HaloWait(self.flags, p.world, p.rank, self.epoch)

    def _enqueue_push(self, local, parity):
        import ctypes
        eng, p = self.engine, self.plan
        eng.bind_stream()
        eng.check(self.lib.sc_halo_push(
            eng.handle, ctypes.c_void_p(local.data_ptr()), self.row_bytes, ctypes.c_void_p(self.src_row.data_ptr()),
            ctypes.c_void_p(self.dst_peer.data_ptr()), ctypes.c_void_p(self.dst_off[parity].data_ptr()),
            int(self.src_row.numel()), ctypes.c_void_p(self.peer_bufs.data_ptr()),
            ctypes.c_void_p(self.peer_flags.data_ptr()), p.world, p.rank, self.epoch), "sc_halo_push")

    def close(self):
        """Collective: unmaps the peers' buffers and frees this rank's buffer."""
        import torch.distributed as dist
        torch.cuda.synchronize(self.engine.device)
        dist.barrier(group=self.group)
        for pp in self.peers.values():
            self.lib.sc_peer_close(self.engine.handle, pp)
        self.peers = {}
        dist.barrier(group=self.group)
        if self.base:
            self.lib.sc_peer_free(self.engine.handle, self.base)
            self.base = 0


def lpt_assign(sizes, world):
    """Greedy longest-processing-time assignment of independent items (batch
    elements of differing voxel counts) to ``world`` ranks: items in
    descending size order, each to the rank with the least total so far (ties
    to the lower rank).  Returns one sorted list of item indices per rank; the
    same on every rank (a pure function of ``sizes``)."""
    order = sorted(range(len(sizes)), key=lambda i: (-int(sizes[i]), i))
    load = [0] * world
    out = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += int(sizes[i])
    return [sorted(x) for x in out]


def batch_rows(coords, batches):
    """Rows of ``coords`` whose batch index is in ``batches``, in input order."""
    b = coords[:, 0].to(torch.int64)
    keep = torch.zeros_like(b, dtype=torch.bool)
    for v in batches:
        keep |= b == int(v)
    return torch.nonzero(keep).squeeze(1)
