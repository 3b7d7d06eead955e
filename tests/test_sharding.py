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


def _pkg_S():
    sys.path.insert(0, ROOT)
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from sparseconv_b200 import sharding as S
    return pkg, S


def test_lpt_assignment():
    _, S = _pkg_S()
    sizes = [40, 55, 31, 60]
    for world in (1, 2, 3, 4, 8):
        a = S.lpt_assign(sizes, world)
        assert len(a) == world
        assert sorted(i for r in a for i in r) == list(range(len(sizes)))  # every item exactly once
        assert a == S.lpt_assign(sizes, world)                            # a pure function of the sizes
    assert S.lpt_assign(sizes, 2) == [[2, 3], [0, 1]]   # 60 -> r0, 55 -> r1, 40 -> r1, 31 -> r0
    assert S.lpt_assign(sizes, 8)[4:] == [[], [], [], []]
    eight = [10] * 8
    assert [sum(eight[i] for i in r) for r in S.lpt_assign(eight, 4)] == [20, 20, 20, 20]


def test_coarsened_partition_keeps_parents_with_their_children():
    pkg, S = _pkg_S()
    w = pkg.workloads.make_workload(4, scale=0.2)
    coords = torch.from_numpy(w.coords)
    parents = torch.unique(torch.stack([coords[:, 0], coords[:, 1] >> 1, coords[:, 2] >> 1, coords[:, 3] >> 1], 1),
                           dim=0)
    for world in (2, 4, 8):
        part = S.MortonPartition.balanced(coords, world)
        coarse = part.coarsen()
        child_owner = part.owner(S.morton_codes(coords))
        par_of_child = torch.stack([coords[:, 0], coords[:, 1] >> 1, coords[:, 2] >> 1, coords[:, 3] >> 1], 1)
        assert torch.equal(coarse.owner(S.morton_codes(par_of_child)), child_owner)
        counts = [int(coarse.owned_rows(parents, r).numel()) for r in range(world)]
        assert sum(counts) == parents.shape[0]


def _chain_worker(rank, world, port):
    """Sharded down -> subm -> up on CPU ranks: the down and up maps of each
    rank's owned fine voxels need no exchange; the coarse subm conv exchanges a
    one-voxel coarse halo (plan without reordering, so local rows are the down
    map's parents in order)."""
    import datetime
    import torch.distributed as dist
    pkg, S = _pkg_S()
    from oracle import sparse_conv_ref as R
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        w = pkg.workloads.make_workload(4, scale=0.15)
        coords = torch.from_numpy(w.coords)
        f = w.feats[:, :16].astype(np.float64)
        rng = np.random.default_rng(9)
        wd = rng.standard_normal((24, 2, 2, 2, 16)) / 11
        ws = rng.standard_normal((24, 3, 3, 3, 24)) / 25
        wu = rng.standard_normal((16, 2, 2, 2, 24)) / 14
        part = S.MortonPartition.balanced(coords, world)
        own = part.owned_rows(coords, rank)
        fine = coords.index_select(0, own).numpy()
        parents, dmap = R.down2_map(fine)
        hd = R.conv_gather(f[own.numpy()], dmap, wd)
        plan = S.build_halo_plan(torch.from_numpy(parents), part.coarsen(), rank, world, interior_first=False)
        assert torch.equal(plan.order, torch.arange(plan.n_own)) and plan.n_interior == 0
        loc = S.exchange_halo(plan, torch.from_numpy(hd))
        loc_c = S.local_coords(plan, torch.from_numpy(parents)).numpy()
        cshape = tuple(s // 2 for s in w.spatial_shape)
        hs = R.conv_gather(loc.numpy(), R.kmap_sorted(loc_c, cshape)[:plan.n_own], ws)
        out = R.conv_gather(hs, R.up2_map(fine, parents), wu)
        # single-rank chain on all voxels
        p_all, d_all = R.down2_map(w.coords)
        hs_all = R.conv_gather(R.conv_gather(f, d_all, wd), R.kmap_sorted(p_all, cshape), ws)
        ref = R.conv_gather(hs_all, R.up2_map(w.coords, p_all), wu)[own.numpy()]
        assert np.allclose(out, ref, rtol=1e-10, atol=1e-10)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_down_subm_up_chain(world):
    mp.spawn(_chain_worker, args=(world, _free_port()), nprocs=world, join=True)


def _dp_worker(rank, world, port):
    """C3-style data parallelism on CPU ranks: batch elements assigned by LPT,
    each rank runs the ResBlock on its elements' rows only, and together they
    reproduce the single-rank result (the map never crosses batch elements)."""
    import datetime
    import torch.distributed as dist
    pkg, S = _pkg_S()
    from oracle import sparse_conv_ref as R
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        w = pkg.workloads.make_workload(3, scale=0.2)
        coords = torch.from_numpy(w.coords)
        sizes = [int((coords[:, 0] == b).sum()) for b in range(w.batch_size)]
        mine = S.lpt_assign(sizes, world)[rank]
        rows = S.batch_rows(coords, mine).numpy()
        f = w.feats[:, :16].astype(np.float64)
        rng = np.random.default_rng(3)
        w1 = rng.standard_normal((16, 3, 3, 3, 16)) / 20
        w2 = rng.standard_normal((16, 3, 3, 3, 16)) / 20
        out = R.resblock(f[rows], R.kmap_sorted(w.coords[rows], w.spatial_shape), w1, None, w2, None)
        ref = R.resblock(f, R.kmap_sorted(w.coords, w.spatial_shape), w1, None, w2, None)[rows]
        assert np.allclose(out, ref, rtol=1e-10, atol=1e-10)
        n = torch.tensor([len(rows)], dtype=torch.int64)
        dist.all_reduce(n)
        assert int(n) == w.n
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_data_parallel_batch_split(world):
    mp.spawn(_dp_worker, args=(world, _free_port()), nprocs=world, join=True)


def _silent_rank_worker(rank, world, port, result_path):
    """Rank 1 builds the plan but never posts its halo send; rank 0's exchange
    must end with an error once the process group's deadline passes, not hang."""
    import datetime
    import time
    import torch.distributed as dist
    pkg, S = _pkg_S()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    w = pkg.workloads.make_workload(1, scale=0.5)
    coords = torch.from_numpy(w.coords)
    part = S.MortonPartition.balanced(coords, world)
    own = part.owned_rows(coords, rank)
    plan = S.build_halo_plan(coords.index_select(0, own).contiguous(), part, rank, world)
    feats = torch.from_numpy(w.feats[:, :8].copy()).index_select(0, S.owned_local(plan, own))
    if rank == 0:
        t0 = time.time()
        try:
            S.exchange_halo(plan, feats)
            outcome = "returned"
        except Exception as e:  # the deadline error of the collective
            outcome = f"raised {type(e).__name__}"
        with open(result_path, "w") as fh:
            fh.write(f"{outcome} {time.time() - t0:.1f}")
    else:
        time.sleep(12)  # never posts its send; leaves after rank 0's deadline
    os._exit(0)  # the group is broken on purpose: leave without its collective teardown


def test_exchange_fails_by_deadline_when_a_rank_never_sends(tmp_path):
    result = tmp_path / "outcome.txt"
    mp.spawn(_silent_rank_worker, args=(2, _free_port(), str(result)), nprocs=2, join=True)
    outcome, seconds = result.read_text().rsplit(" ", 1)
    assert outcome.startswith("raised"), outcome
    assert float(seconds) < 30.0
