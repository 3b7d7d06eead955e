"""Kernel-map parity on the GPU: bit-exact against the CPU oracle."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _coords(w, cuda, perm=None):
    c = w.coords if perm is None else w.coords[perm]
    return torch.from_numpy(np.ascontiguousarray(c)).to(cuda)


@pytest.mark.parametrize("cfg,scale", [(1, 1.0), (2, 0.3), (3, 0.4)])
@pytest.mark.parametrize("mode", ["hash", "sort"])
def test_subm_map_bit_exact(pkg, oracle, cuda, cfg, scale, mode):
    w = pkg.workloads.make_workload(cfg, scale=scale)
    perm = pkg.workloads.shuffle_rows(w.n, cfg)
    coords = w.coords[perm]
    ref = oracle.kmap_sorted(coords, w.spatial_shape)
    if cfg == 1:
        assert np.array_equal(ref, oracle.kmap_bruteforce(coords, w.spatial_shape, w.batch_size))
    km = pkg.build_kmap(_coords(w, cuda, perm), engine=pkg.get_engine(cuda, mode))
    got = km.export().cpu().numpy()
    assert np.array_equal(got, ref)
    info = km.info()
    assert info["num_pairs"] == int((ref >= 0).sum())
    assert info["n_out"] == w.n and info["kernel_volume"] == 27


@pytest.mark.parametrize("dil", [2, 3])
def test_dilated_map(pkg, oracle, cuda, dil):
    w = pkg.workloads.make_workload(1)
    ref = oracle.kmap_bruteforce(w.coords, w.spatial_shape, 1, dilation=dil)
    got = pkg.build_kmap(_coords(w, cuda), dilation=dil).export().cpu().numpy()
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("dil", [(1, 2, 3), (2, 1, 1)])
def test_anisotropic_dilation_map(pkg, oracle, cuda, dil):
    """Per-axis dilation (the reference's dilD, dilH, dilW; kd on x), full and range builds."""
    w = pkg.workloads.make_workload(1)
    ref = oracle.kmap_bruteforce(w.coords, w.spatial_shape, 1, dilation=dil)
    c = _coords(w, cuda)
    for mode in ("hash", "sort"):
        got = pkg.build_kmap(c, dilation=dil, engine=pkg.get_engine(cuda, mode)).export().cpu().numpy()
        assert np.array_equal(got, ref), mode
    lo, hi = w.n // 3, (2 * w.n) // 3
    got = pkg.build_kmap(c, dilation=dil, out_begin=lo, n_out=hi - lo).export().cpu().numpy()
    assert np.array_equal(got, ref[lo:hi])


def test_sparse_conv3d_anisotropic_dilation(pkg, oracle, cuda):
    w = pkg.workloads.make_workload(2, scale=0.2)
    c = _coords(w, cuda)
    rng = np.random.default_rng(12)
    f = torch.from_numpy(rng.standard_normal((w.n, 64)).astype(np.float32)).to(cuda, torch.bfloat16)
    W = torch.from_numpy((rng.standard_normal((64, 3, 3, 3, 64)) / 40).astype(np.float32)).to(cuda, torch.bfloat16)
    conv = pkg.SparseConv3d(W, dilation=(2, 1, 3))
    y = conv(pkg.SparseTensor(f, c))
    assert conv.cache_key() == "conv_neighbors_3x3x3_dil3x1x2"
    ref = oracle.conv_gather(f.float().cpu().numpy(), oracle.kmap_sorted(w.coords, w.spatial_shape, (2, 1, 3)),
                             W.float().cpu().numpy())
    out = y.feats.float().cpu().numpy()
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 5e-3


def test_tile_sort_does_not_change_map(pkg, cuda):
    w = pkg.workloads.make_workload(2, scale=0.3)
    c = _coords(w, cuda)
    a = pkg.build_kmap(c, tile_sort=True)
    b = pkg.build_kmap(c, tile_sort=False)
    assert torch.equal(a.export(), b.export())
    ia, ib = a.info(), b.info()
    assert ia["num_pairs"] == ib["num_pairs"]
    assert ia["tile_pairs"] <= ib["tile_pairs"]


def test_batch_index_is_part_of_the_key(pkg, oracle, cuda):
    # the same spatial coords in two batch entries never see each other
    w = pkg.workloads.make_workload(1, scale=0.5)
    c2 = np.concatenate([w.coords, w.coords.copy()], 0)
    c2[w.n:, 0] = 1
    ref = oracle.kmap_bruteforce(c2, w.spatial_shape, 2)
    got = pkg.build_kmap(torch.from_numpy(c2).to(cuda)).export().cpu().numpy()
    assert np.array_equal(got, ref)
    assert (got[:w.n][got[:w.n] >= 0] < w.n).all() and (got[w.n:][got[w.n:] >= 0] >= w.n).all()


def test_edges_small_inputs(pkg, oracle, cuda):
    # empty, one voxel, voxels at the corners of the coordinate range
    km = pkg.build_kmap(torch.zeros((0, 4), dtype=torch.int32, device=cuda))
    assert km.export().shape == (0, 27)
    one = torch.tensor([[0, 5, 5, 5]], dtype=torch.int32, device=cuda)
    m = pkg.build_kmap(one).export().cpu().numpy()
    assert m[0, 13] == 0 and (np.delete(m[0], 13) == -1).all()
    corners = np.array([[0, 0, 0, 0], [0, 0, 0, 1], [0, 65535, 65535, 65535], [0, 65534, 65535, 65535],
                        [32767, 0, 0, 0], [32767, 65535, 65535, 65535]], np.int32)
    got = pkg.build_kmap(torch.from_numpy(corners).to(cuda)).export().cpu().numpy()
    assert np.array_equal(got, oracle.kmap_sorted(corners, (65536, 65536, 65536)))


def test_ragged_tile_counts(pkg, oracle, cuda):
    # N not a multiple of the 128-row tile nor of the 2048-key sort tile
    w = pkg.workloads.make_workload(1)
    for n in (1, 127, 129, 2047, 2049, 4097):
        c = np.ascontiguousarray(w.coords[:n])
        ref = oracle.kmap_sorted(c, w.spatial_shape)
        for mode in ("hash", "sort"):
            got = pkg.build_kmap(torch.from_numpy(c).to(cuda), engine=pkg.get_engine(cuda, mode)).export()
            assert np.array_equal(got.cpu().numpy(), ref), (n, mode)


def test_duplicate_coords_raise(pkg, cuda):
    w = pkg.workloads.make_workload(1)
    c = np.concatenate([w.coords, w.coords[100:101]], 0)
    for mode in ("hash", "sort"):
        with pytest.raises(pkg.DuplicateCoordError):
            pkg.build_kmap(torch.from_numpy(c).to(cuda), engine=pkg.get_engine(cuda, mode))
    with pytest.raises(pkg.DuplicateCoordError):
        pkg.build_down2(torch.from_numpy(c).to(cuda))


def test_out_of_range_coords_raise(pkg, cuda):
    for bad in ([0, -1, 3, 3], [0, 3, 65536, 3], [-2, 1, 1, 1], [32768, 1, 1, 1]):
        c = torch.tensor([[0, 1, 1, 1], bad], dtype=torch.int32, device=cuda)
        for mode in ("hash", "sort"):
            with pytest.raises(pkg.CoordRangeError):
                pkg.build_kmap(c, engine=pkg.get_engine(cuda, mode))
        with pytest.raises(pkg.CoordRangeError):
            pkg.build_down2(c)


def test_engine_usable_after_errors(pkg, oracle, cuda):
    w = pkg.workloads.make_workload(1)
    bad = torch.tensor([[0, -5, 0, 0]], dtype=torch.int32, device=cuda)
    with pytest.raises(pkg.CoordRangeError):
        pkg.build_kmap(bad)
    got = pkg.build_kmap(_coords(w, cuda)).export().cpu().numpy()
    assert np.array_equal(got, oracle.kmap_sorted(w.coords, w.spatial_shape))


@pytest.mark.parametrize("cfg,scale", [(1, 1.0), (4, 0.2), (3, 0.4)])
def test_down_up_maps(pkg, oracle, cuda, cfg, scale):
    w = pkg.workloads.make_workload(cfg, scale=scale)
    perm = pkg.workloads.shuffle_rows(w.n, cfg)
    coords = np.ascontiguousarray(w.coords[perm])
    pc_ref, dmap_ref = oracle.down2_map(coords)
    down = pkg.build_down2(torch.from_numpy(coords).to(cuda))
    assert np.array_equal(down.out_coords().cpu().numpy(), pc_ref)
    assert np.array_equal(down.export().cpu().numpy(), dmap_ref)
    up = pkg.build_up2(down)
    assert np.array_equal(up.export().cpu().numpy(), oracle.up2_map(coords, pc_ref))
    assert up.info()["num_pairs"] == w.n


def test_full_size_c2_map(pkg, oracle, cuda):
    w = pkg.workloads.make_workload(2)
    ref = oracle.kmap_sorted(w.coords, w.spatial_shape)
    for mode in ("hash", "sort"):
        got = pkg.build_kmap(_coords(w, cuda), engine=pkg.get_engine(cuda, mode)).export().cpu().numpy()
        assert np.array_equal(got, ref), mode


def test_full_size_c5_map(pkg, oracle, cuda):
    # the oracle's torch-CPU sort + searchsorted (multithreaded; equal to
    # kmap_sorted, tests/test_oracle.py) keeps the 6.1M-voxel check in seconds
    w = pkg.workloads.make_workload(5)
    ref = oracle.torch_cpu_kmap(torch.from_numpy(w.coords), w.spatial_shape).numpy()
    got = pkg.build_kmap(_coords(w, cuda)).export().cpu().numpy()
    assert np.array_equal(got, ref)
    got_sort = pkg.build_kmap(_coords(w, cuda), engine=pkg.get_engine(cuda, "sort")).export().cpu().numpy()
    assert np.array_equal(got_sort, ref)


def test_map_build_is_deterministic(pkg, cuda):
    w = pkg.workloads.make_workload(3, scale=0.4)
    c = _coords(w, cuda)
    a = pkg.build_kmap(c)
    b = pkg.build_kmap(c)
    assert torch.equal(a.export(), b.export())


def test_map_with_fewer_outputs(pkg, oracle, cuda):
    # outputs are the first n_out rows, neighbours come from all rows (sharded convs)
    w = pkg.workloads.make_workload(3, scale=0.3)
    perm = pkg.workloads.shuffle_rows(w.n, 3)
    coords = np.ascontiguousarray(w.coords[perm])
    ref = oracle.kmap_sorted(coords, w.spatial_shape)
    c = torch.from_numpy(coords).to(cuda)
    for n_out in (0, 1, 777, w.n // 2, w.n):
        for mode in ("hash", "sort"):
            km = pkg.build_kmap(c, n_out=n_out, engine=pkg.get_engine(cuda, mode))
            assert km.n_out == n_out and km.n_in == w.n
            assert np.array_equal(km.export().cpu().numpy(), ref[:n_out]), (n_out, mode)


def test_range_build_equals_full_map_rows(pkg, oracle, cuda):
    # outputs = rows [a, b) (sc_kmap_build_range); neighbours from all rows
    w = pkg.workloads.make_workload(2, scale=0.25)
    c = torch.from_numpy(w.coords).to(cuda)
    full = oracle.kmap_sorted(w.coords, w.spatial_shape)
    a, b = w.n // 3, w.n // 3 + 777
    km = pkg.build_kmap(c, out_begin=a, n_out=b - a)
    assert km.n_out == b - a and km.n_in == w.n
    assert np.array_equal(km.export().cpu().numpy(), full[a:b])
    km_tail = pkg.build_kmap(c, out_begin=b)
    assert np.array_equal(km_tail.export().cpu().numpy(), full[b:])
