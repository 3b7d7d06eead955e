"""Morton-range sharded conv on 2+ GPUs against one GPU.

Each rank owns a Morton range, exchanges its halo (all_to_all_single over
NCCL; the library's peer-memory push followed by its wait kernel or by a conv
that waits inside its kernel), builds its map with owned rows as outputs, and
runs the tcgen05 conv.
Owned outputs must equal the single-GPU conv bit for bit: every output row
sums the same offsets in the same order, and offsets a tile skips add zeros.
Skipped unless at least two GPUs are visible.
"""
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, cfg, scale, ch):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from sparseconv_b200 import sharding as S
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        w = pkg.workloads.make_workload(cfg, scale=scale)
        coords = torch.from_numpy(w.coords).to(dev)
        feats = torch.from_numpy(w.feats[:, :ch].copy()).to(dev, torch.bfloat16)
        W = torch.from_numpy(w.weight[:ch, :, :, :, :ch].copy()).to(dev, torch.bfloat16)
        ref = pkg.conv3d(pkg.build_kmap(coords), feats, W)  # whole problem on this GPU
        part = S.MortonPartition.balanced(coords, world)
        own = part.owned_rows(coords, rank)
        own_c = coords.index_select(0, own).contiguous()
        plan = S.build_halo_plan(own_c, part, rank, world)
        own = S.owned_local(plan, own)  # global row of each local owned row
        loc_c = S.local_coords(plan, own_c)
        loc_f = S.exchange_halo(plan, feats.index_select(0, own))
        km = pkg.build_kmap(loc_c, n_out=plan.n_own)
        out = pkg.conv3d(km, loc_f, W)
        torch.cuda.synchronize()
        assert out.shape == (plan.n_own, ch)
        assert torch.equal(out, ref.index_select(0, own))
        # interior outputs while the halo is in flight, then boundary outputs
        ni = plan.n_interior
        km_i = pkg.build_kmap(loc_c, n_out=ni)
        km_b = pkg.build_kmap(loc_c, out_begin=ni, n_out=plan.n_own - ni)
        buf = torch.zeros_like(loc_f)
        buf[:plan.n_own].copy_(feats.index_select(0, own))
        split = torch.empty_like(out)
        eng = pkg.get_engine(dev)
        eng.set_conv_ctas(torch.cuda.get_device_properties(dev).multi_processor_count - 16)
        _, work = S.exchange_halo(plan, buf[:plan.n_own], out=buf, async_op=True)
        pkg.conv3d(km_i, buf, W, out=split[:ni])
        work.wait()
        eng.set_conv_ctas(0)
        pkg.conv3d(km_b, buf, W, out=split[ni:])
        torch.cuda.synchronize()
        assert torch.equal(split, out)
        # halo exchange over peer memory (IPC buffers, push + wait kernels) equals NCCL's
        px = S.PeerHaloExchange(plan, feats.index_select(0, own), eng)
        for _ in range(3):  # both regions, twice for the first
            loc = px.exchange()
            out_p = pkg.conv3d(km, loc, W)
            torch.cuda.synchronize()
            assert torch.equal(loc, loc_f)
            assert torch.equal(out_p, out)
        # push only; the conv on the interior+boundary map waits in its kernel
        km_c = pkg.concat_kmaps(km_i, km_b)
        for _ in range(4):
            loc, hw = px.push()
            out_c = pkg.conv3d(km_c, loc, W, halo_wait=hw)
            torch.cuda.synchronize()
            assert torch.equal(loc, loc_f)
            assert torch.equal(out_c, out)
        # back-to-back layers without host synchronisation
        outs = []
        for _ in range(6):
            loc, hw = px.push()
            outs.append(pkg.conv3d(km_c, loc, W, halo_wait=hw))
        torch.cuda.synchronize()
        for o in outs:
            assert torch.equal(o, out)
        eng.synchronize()  # no device wait timed out
        px.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("cfg,scale,ch", [(2, 0.4, 128), (5, 0.2, 32), (3, 0.3, 64)])
def test_sharded_conv_equals_single_gpu(cfg, scale, ch):
    world = min(torch.cuda.device_count(), 4)
    mp.spawn(_worker, args=(world, _free_port(), cfg, scale, ch), nprocs=world, join=True)
