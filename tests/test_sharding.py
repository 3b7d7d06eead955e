"""Morton-range sharding + halo exchange on CPU ranks (gloo), checked against one rank.

Each rank owns a Morton range of the voxels, builds its halo plan, exchanges
features with all_to_all_single, and runs the oracle conv on owned + halo
rows.  Owned outputs must equal the single-rank result: the neighbour map
bit-exactly (after translating local rows to global rows) and the conv to f32
rounding.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, cfg, scale):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from oracle import sparse_conv_ref as R
    from sparseconv_b200 import sharding as S
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        w = pkg.workloads.make_workload(cfg, scale=scale)
        coords = torch.from_numpy(w.coords)
        part = S.MortonPartition.balanced(coords, world)
        # boundaries are multiples of 8: every 2x2x2 sibling group is on one rank
        for b in part.bounds[1:-1].tolist():
            assert b % 8 == 0
        own = part.owned_rows(coords, rank)
        own_coords = coords.index_select(0, own).contiguous()
        plan = S.build_halo_plan(own_coords, part, rank, world)
        own = S.owned_local(plan, own)  # global row of each local owned row
        assert torch.equal(torch.sort(own).values, part.owned_rows(coords, rank))
        feats = torch.from_numpy(w.feats[:, :16].copy())
        loc_f = S.exchange_halo(plan, feats.index_select(0, own))
        loc_c = S.local_coords(plan, own_coords)
        # halo rows carry the right features
        gkeys = R.flat_keys(w.coords, w.spatial_shape)
        order = np.argsort(gkeys)
        lk = R.flat_keys(loc_c.numpy(), w.spatial_shape)
        gid = order[np.searchsorted(gkeys[order], lk)]
        assert np.array_equal(gkeys[gid], lk)
        assert torch.equal(loc_f, feats.index_select(0, torch.from_numpy(gid)))
        # owned map rows (translated to global rows) equal the global map
        km_loc = R.kmap_sorted(loc_c.numpy(), w.spatial_shape)[:plan.n_own]
        km_glob = R.kmap_sorted(w.coords, w.spatial_shape)[own.numpy()]
        translated = np.where(km_loc >= 0, gid[np.maximum(km_loc, 0)], -1)
        assert np.array_equal(translated, km_glob)
        # interior rows (first in plan order) read no halo row; some rows are interior
        assert (km_loc[:plan.n_interior] < plan.n_own).all()
        assert 0 < plan.n_interior <= plan.n_own
        # owned conv outputs equal the single-rank conv
        W = torch.from_numpy(w.weight[:16, :, :, :, :16].copy())
        out = R.torch_cpu_conv(loc_f, torch.from_numpy(km_loc), W)
        ref = R.conv_gather(feats.numpy(), R.kmap_sorted(w.coords, w.spatial_shape), W.numpy())[own.numpy()]
        rel = np.linalg.norm(out.numpy() - ref) / np.linalg.norm(ref)
        assert rel < 1e-6, rel
        # every voxel is owned by exactly one rank
        cnt = torch.tensor([plan.n_own], dtype=torch.int64)
        dist.all_reduce(cnt)
        assert int(cnt) == w.n
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_halo_exchange_matches_single_rank(world):
    mp.spawn(_worker, args=(world, _free_port(), 1, 1.0), nprocs=world, join=True)


def test_halo_exchange_multi_batch():
    mp.spawn(_worker, args=(3, _free_port(), 3, 0.25), nprocs=3, join=True)


def test_partition_is_balanced_and_aligned():
    sys.path.insert(0, ROOT)
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from sparseconv_b200 import sharding as S
    w = pkg.workloads.make_workload(2, scale=0.3)
    coords = torch.from_numpy(w.coords)
    for world in (2, 4, 8):
        part = S.MortonPartition.balanced(coords, world)
        counts = [int(part.owned_rows(coords, r).numel()) for r in range(world)]
        assert sum(counts) == w.n
        assert max(counts) - min(counts) <= max(64, w.n // 50)
        codes = S.morton_codes(coords)
        owner = part.owner(codes)
        # siblings (same code >> 3) never straddle ranks
        parent = codes >> 3
        for r in range(world):
            sib = parent[owner == r]
            assert not torch.isin(sib, parent[owner != r]).any()


def _peer_worker(rank, world, port, cfg, scale):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from sparseconv_b200 import sharding as S
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        w = pkg.workloads.make_workload(cfg, scale=scale)
        coords = torch.from_numpy(w.coords)
        part = S.MortonPartition.balanced(coords, world)
        own = part.owned_rows(coords, rank)
        own_c = coords.index_select(0, own).contiguous()
        plan = S.build_halo_plan(own_c, part, rank, world)
        infos = [None] * world
        dist.all_gather_object(infos, (plan.n_own, list(plan.recv_splits)))
        dst_peer, dst_row = S.peer_destinations(plan, infos)
        # what every rank writes where: (dest rank, dest row, coords of the row written)
        local = S.local_coords(plan, own_c)
        sent = [(p, r, tuple(local[int(i)].tolist())) for p, r, i in zip(dst_peer, dst_row, plan.send_idx.tolist())]
        allsent = [None] * world
        dist.all_gather_object(allsent, sent)
        # rows written into this rank's buffer tile its halo region exactly, with the plan's halo coords
        mine = sorted((r, c) for lst in allsent for (p, r, c) in lst if p == rank)
        assert [r for r, _ in mine] == list(range(plan.n_own, plan.n_own + plan.n_halo))
        for r, c in mine:
            assert tuple(local[r].tolist()) == c
        # a plan that disagrees on the counts is refused
        if plan.send_splits[(rank + 1) % world] > 0:
            bad = list(infos)
            s = (rank + 1) % world
            bad[s] = (infos[s][0], [x + 1 for x in infos[s][1]])
            try:
                S.peer_destinations(plan, bad)
                raise AssertionError("mismatched plan accepted")
            except RuntimeError:
                pass
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_peer_destinations_tile_every_halo(world):
    mp.spawn(_peer_worker, args=(world, _free_port(), 2, 0.3), nprocs=world, join=True)
