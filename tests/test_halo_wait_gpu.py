"""Concatenated maps (sc_kmap_concat) and convs that wait on the device for a
halo exchange (sc_conv3d_halo), on one GPU.

The exchange's flag words are a device array the test writes: flags already
at the epoch let the conv run through, and its results must equal the plain
conv's bit for bit (tiles a wait delays compute the same sums).  Flags that
never reach the epoch make the kernel's bounded wait run out: the conv still
completes, the next synchronize reports SC_ETIMEOUT, and the context stays
usable.  A concatenated map waits only before its second part, and at the
latest before the kernel ends.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(pkg, cuda, cfg, scale, ci, co, dtype=torch.bfloat16, seed=0):
    w = pkg.workloads.make_workload(cfg, scale=scale)
    rng = np.random.default_rng(seed)
    f = torch.from_numpy(rng.standard_normal((w.n, ci)).astype(np.float32)).to(cuda, dtype)
    W = torch.from_numpy((rng.standard_normal((co, 3, 3, 3, ci)) / np.sqrt(27 * ci)).astype(np.float32)).to(cuda, dtype)
    b = torch.from_numpy((0.1 * rng.standard_normal(co)).astype(np.float32)).to(cuda, dtype)
    return torch.from_numpy(w.coords).to(cuda), f, W, b


def _flags(cuda, values):
    """Device array of uint32 flag words (stored as int32)."""
    return torch.from_numpy(np.array(values, np.uint64).astype(np.uint32).view(np.int32)).to(cuda)


@pytest.mark.parametrize("split_frac", [0.0, 0.37, 0.9, 1.0])
def test_concat_map_equals_parts(pkg, cuda, split_frac):
    c, f, W, b = _inputs(pkg, cuda, 2, 0.3, 64, 64)
    n = c.shape[0]
    split = int(n * split_frac)
    km_a = pkg.build_kmap(c, n_out=split)
    km_b = pkg.build_kmap(c, out_begin=split, n_out=n - split)
    km = pkg.concat_kmaps(km_a, km_b)
    whole = pkg.build_kmap(c)
    assert km.n_out == n
    assert torch.equal(km.export(), torch.cat([km_a.export(), km_b.export()]))
    assert torch.equal(km.export(), whole.export())
    ia, ib, ic = km_a.info(), km_b.info(), km.info()
    assert ic["num_tiles"] == ia["num_tiles"] + ib["num_tiles"]
    assert ic["num_pairs"] == ia["num_pairs"] + ib["num_pairs"] == whole.info()["num_pairs"]
    assert ic["tile_pairs"] == ia["tile_pairs"] + ib["tile_pairs"]
    assert ic["halo_max"] == -1
    out = pkg.conv3d(km, f, W, b)
    torch.cuda.synchronize()
    assert torch.equal(out, pkg.conv3d(whole, f, W, b))


def test_concat_rejects_mismatched_maps(pkg, cuda):
    c, _, _, _ = _inputs(pkg, cuda, 1, 0.3, 16, 16)
    km = pkg.build_kmap(c)
    down = pkg.build_down2(c)
    with pytest.raises(ValueError):
        pkg.concat_kmaps(km, down)
    other = pkg.build_kmap(c[: c.shape[0] // 2].contiguous())
    with pytest.raises(ValueError):
        pkg.concat_kmaps(km, other)


@pytest.mark.parametrize("ci,co,dtype", [(32, 32, torch.bfloat16), (128, 128, torch.bfloat16),
                                         (64, 48, torch.float16), (32, 32, torch.float32)])
def test_conv_after_arrived_exchange_equals_plain(pkg, cuda, ci, co, dtype):
    c, f, W, b = _inputs(pkg, cuda, 2, 0.3, ci, co, dtype=dtype, seed=1)
    n = c.shape[0]
    split = (n * 3) // 4 + 5
    km = pkg.concat_kmaps(pkg.build_kmap(c, n_out=split), pkg.build_kmap(c, out_begin=split, n_out=n - split))
    whole = pkg.build_kmap(c)
    ref = pkg.conv3d(whole, f, W, b, silu=True)
    eng = pkg.get_engine(cuda)
    # world 4, rank 1: words 0, 2, 3 count; word 1 (this rank) is never read
    cases = [([7, 0, 7, 9], 7), ([3, 0, 5, 4], 3), ([1, 0, 2, 0xFFFFFFFF], 0xFFFFFFFF)]  # last: epoch wraps
    for vals, epoch in cases:
        flags = _flags(cuda, vals)
        hw = pkg.HaloWait(flags.data_ptr(), 4, 1, epoch)
        out_c = pkg.conv3d(km, f, W, b, silu=True, halo_wait=hw)
        out_w = pkg.conv3d(whole, f, W, b, silu=True, halo_wait=hw)
        eng.synchronize()
        assert torch.equal(out_c, ref)
        assert torch.equal(out_w, ref)


def test_conv_wait_times_out_and_context_survives(pkg, cuda):
    c, f, W, b = _inputs(pkg, cuda, 2, 0.25, 32, 32, seed=2)
    n = c.shape[0]
    split = n // 2
    whole = pkg.build_kmap(c)
    ref = pkg.conv3d(whole, f, W, b)
    eng = pkg.get_engine(cuda)
    eng.synchronize()
    flags = _flags(cuda, [5, 5, 5])  # never reaches epoch 6
    hw = pkg.HaloWait(flags.data_ptr(), 3, 0, 6)
    maps = {
        "plain": whole,  # waits before its first tile
        "concat": pkg.concat_kmaps(pkg.build_kmap(c, n_out=split), pkg.build_kmap(c, out_begin=split,
                                                                                   n_out=n - split)),
        "no second part": pkg.concat_kmaps(pkg.build_kmap(c, n_out=n), pkg.build_kmap(c, out_begin=n, n_out=0)),
    }
    for name, km in maps.items():
        out = pkg.conv3d(km, f, W, b, halo_wait=hw)
        with pytest.raises(pkg.SparseConvError) as ei:
            eng.synchronize()
        assert ei.value.status == pkg._lib.SC_ETIMEOUT, name
        # every row was still computed (all rows are local here)
        assert torch.equal(out, ref), name
    # the error was reported once; the next conv runs normally
    out = pkg.conv3d(whole, f, W, b)
    eng.synchronize()
    assert torch.equal(out, ref)
