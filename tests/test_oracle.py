"""CPU checks of the oracle restatement (no GPU).

The reference documents two invariants for its sparse-conv path
(README.md:80-81): the neighbour lookup equals brute force, and the sparse
conv equals dense F.conv3d to 1e-5.  These tests establish both for the
oracle, then pin it to the committed golden fixtures.
"""
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("cfg,scale", [(1, 1.0), (1, 0.5), (3, 0.3)])
def test_sorted_map_equals_bruteforce(pkg, oracle, cfg, scale):
    w = pkg.workloads.make_workload(cfg, scale=scale)
    perm = pkg.workloads.shuffle_rows(w.n, cfg)
    c = w.coords[perm]
    a = oracle.kmap_bruteforce(c, w.spatial_shape, w.batch_size)
    b = oracle.kmap_sorted(c, w.spatial_shape)
    assert np.array_equal(a, b)
    # centre column is the row itself; symmetric offsets are inverse maps
    assert np.array_equal(a[:, 13], np.arange(len(c)))
    for v in range(27):
        rows = np.where(a[:, v] >= 0)[0]
        assert np.array_equal(a[a[rows, v], 26 - v], rows)


def test_torch_cpu_map_equals_numpy(pkg, oracle):
    w = pkg.workloads.make_workload(1)
    a = oracle.kmap_sorted(w.coords, w.spatial_shape)
    b = oracle.torch_cpu_kmap(torch.from_numpy(w.coords), w.spatial_shape).numpy()
    assert np.array_equal(a, b)


def test_dilated_map(pkg, oracle):
    w = pkg.workloads.make_workload(1, scale=0.6)
    for d in (2, 3):
        assert np.array_equal(oracle.kmap_bruteforce(w.coords, w.spatial_shape, 1, d),
                              oracle.kmap_sorted(w.coords, w.spatial_shape, d))
    # per-axis dilation (dilD on x, dilH on y, dilW on z) and map-row subsets
    for d in ((1, 2, 3), (3, 1, 2)):
        full = oracle.kmap_bruteforce(w.coords, w.spatial_shape, 1, d)
        assert np.array_equal(full, oracle.kmap_sorted(w.coords, w.spatial_shape, d))
        rows = np.random.default_rng(1).choice(w.n, 500, replace=False)
        assert np.array_equal(full[rows], oracle.kmap_sorted(w.coords, w.spatial_shape, d, rows=rows))
    off = oracle.offsets27((1, 2, 3))
    assert off[0].tolist() == [-1, -2, -3] and off[26].tolist() == [1, 2, 3] and off[13].tolist() == [0, 0, 0]


def test_round_bf16_matches_torch(oracle):
    x = np.random.default_rng(2).standard_normal(50000) * 37.0
    ref = torch.from_numpy(x).float().to(torch.bfloat16).double().numpy()
    assert np.array_equal(oracle.round_bf16(x), ref)


def test_duplicates_rejected(pkg, oracle):
    w = pkg.workloads.make_workload(1, scale=0.5)
    c = np.concatenate([w.coords, w.coords[:1]], 0)
    with pytest.raises(ValueError):
        oracle.kmap_sorted(c, w.spatial_shape)
    with pytest.raises(ValueError):
        oracle.kmap_bruteforce(c, w.spatial_shape, 1)


def test_conv_matches_dense_conv3d(pkg, oracle):
    w = pkg.workloads.make_workload(1)
    rng = np.random.default_rng(3)
    f = rng.standard_normal((w.n, 8)).astype(np.float32)
    W = (rng.standard_normal((8, 3, 3, 3, 8)) / 14).astype(np.float32)
    b = (0.1 * rng.standard_normal(8)).astype(np.float32)
    km = oracle.kmap_sorted(w.coords, w.spatial_shape)
    sparse = oracle.conv_gather(f, km, W, b)
    dense = oracle.dense_conv3d_check(w.coords, f, W, b, w.spatial_shape, 1)
    assert rel_l2(sparse, dense) < 1e-12  # both float64
    # torch-CPU f32 version used for the CPU baseline
    t = oracle.torch_cpu_conv(torch.from_numpy(f), torch.from_numpy(km), torch.from_numpy(W), torch.from_numpy(b))
    assert rel_l2(t.numpy(), dense) < 1e-5


def test_down_conv_matches_strided_dense(pkg, oracle):
    w = pkg.workloads.make_workload(4, scale=0.04)
    rng = np.random.default_rng(5)
    f = rng.standard_normal((w.n, 4)).astype(np.float64)
    W = rng.standard_normal((6, 2, 2, 2, 4))
    pc, dmap = oracle.down2_map(w.coords)
    sparse = oracle.conv_gather(f, dmap, W)
    c = torch.as_tensor(w.coords.astype(np.int64))
    X = int(c[:, 1:].max()) + 2
    X += X % 2
    dense = torch.zeros((1, 4, X, X, X), dtype=torch.float64)
    dense[c[:, 0], :, c[:, 1], c[:, 2], c[:, 3]] = torch.as_tensor(f)
    y = F.conv3d(dense, torch.as_tensor(W).permute(0, 4, 1, 2, 3), stride=2)
    p = torch.as_tensor(pc.astype(np.int64))
    ref = y[p[:, 0], :, p[:, 1], p[:, 2], p[:, 3]].numpy()
    assert rel_l2(sparse, ref) < 1e-12
    # parents are unique and in ascending lexicographic order
    keys = ((pc[:, 0].astype(np.int64) * 65536 + pc[:, 1]) * 65536 + pc[:, 2]) * 65536 + pc[:, 3]
    assert np.all(np.diff(keys) > 0)


def test_up_conv_matches_transposed_dense(pkg, oracle):
    w = pkg.workloads.make_workload(4, scale=0.04)
    rng = np.random.default_rng(6)
    pc, _ = oracle.down2_map(w.coords)
    g = rng.standard_normal((len(pc), 5))
    W = rng.standard_normal((3, 2, 2, 2, 5))
    umap = oracle.up2_map(w.coords, pc)
    sparse = oracle.conv_gather(g, umap, W)
    p = torch.as_tensor(pc.astype(np.int64))
    Xc = int(p[:, 1:].max()) + 1
    dense = torch.zeros((1, 5, Xc, Xc, Xc), dtype=torch.float64)
    dense[p[:, 0], :, p[:, 1], p[:, 2], p[:, 3]] = torch.as_tensor(g)
    y = F.conv_transpose3d(dense, torch.as_tensor(W).permute(4, 0, 1, 2, 3), stride=2)
    c = torch.as_tensor(w.coords.astype(np.int64))
    ref = y[c[:, 0], :, c[:, 1], c[:, 2], c[:, 3]].numpy()
    assert rel_l2(sparse, ref) < 1e-12
    assert np.all((umap >= 0).sum(1) == 1)


def test_layernorm_silu_match_torch(oracle):
    x = np.random.default_rng(1).standard_normal((50, 32))
    ln = torch.nn.functional.layer_norm(torch.as_tensor(x), (32,), eps=1e-6).numpy()
    assert rel_l2(oracle.layer_norm(x, 1e-6), ln) < 1e-12
    assert rel_l2(oracle.silu(x), torch.nn.functional.silu(torch.as_tensor(x)).numpy()) < 1e-12


def test_golden_fixtures_pin_the_oracle(oracle):
    d = np.load(os.path.join(GOLDEN, "subm_c1_small.npz"))
    shape = tuple(d["spatial_shape"])
    km = oracle.kmap_sorted(d["coords"], shape)
    assert np.array_equal(km, d["kmap"])
    assert np.array_equal(km, oracle.kmap_bruteforce(d["coords"], shape, 1))
    assert np.array_equal(oracle.kmap_sorted(d["coords"], shape, 2), d["kmap_dil2"])
    assert rel_l2(oracle.conv_gather(d["feats"], km, d["weight"], d["bias"]), d["out"]) < 1e-6
    d2 = np.load(os.path.join(GOLDEN, "subm_batch2.npz"))
    assert np.array_equal(oracle.kmap_bruteforce(d2["coords"], (64, 64, 64), 2), d2["kmap"])
    d3 = np.load(os.path.join(GOLDEN, "downup_c4_small.npz"))
    pc, dmap = oracle.down2_map(d3["coords"])
    assert np.array_equal(pc, d3["parent_coords"]) and np.array_equal(dmap, d3["dmap"])
    assert np.array_equal(oracle.up2_map(d3["coords"], pc), d3["umap"])
    assert rel_l2(oracle.conv_gather(d3["feats"], dmap, d3["w_down"]), d3["out_down"]) < 1e-6


def test_workloads_are_deterministic_and_valid(pkg):
    for cfg, scale in [(1, 1.0), (2, 0.2), (3, 0.2), (4, 0.05)]:
        a = pkg.workloads.make_workload(cfg, scale=scale)
        b = pkg.workloads.make_workload(cfg, scale=scale)
        assert np.array_equal(a.coords, b.coords) and np.array_equal(a.feats, b.feats)
        c = a.coords.astype(np.int64)
        key = ((c[:, 0] * 65536 + c[:, 1]) * 65536 + c[:, 2]) * 65536 + c[:, 3]
        assert len(np.unique(key)) == len(c)
        assert c.min() >= 0 and c[:, 1:].max() < a.spatial_shape[0]
        assert np.all(np.diff(c[:, 0]) >= 0)  # batch-sorted


def test_depthwise_oracle_is_dense_conv_with_diagonal_weight(oracle):
    rng = np.random.default_rng(21)
    coords = np.unique(rng.integers(0, 12, (300, 3)), axis=0)
    coords = np.concatenate([np.zeros((len(coords), 1), np.int64), coords], 1).astype(np.int32)
    km = oracle.kmap_sorted(coords, (12, 12, 12))
    c = 5
    f = rng.standard_normal((len(coords), c))
    wd = rng.standard_normal((c, 3, 3, 3, 1))
    b = rng.standard_normal(c)
    dense = np.zeros((c, 27, c))
    dense[np.arange(c), :, np.arange(c)] = wd.reshape(c, 27)
    np.testing.assert_allclose(oracle.conv_depthwise(f, km, wd, b), oracle.conv_gather(f, km, dense, b), rtol=1e-12)


def test_convnext_block_oracle_matches_torch(oracle):
    """The block against torch.nn.functional in float64 (dense conv through
    the dense-grid check, LayerNorm without affine, eps 1e-6)."""
    import torch
    import torch.nn.functional as F
    rng = np.random.default_rng(22)
    coords = np.unique(rng.integers(0, 10, (250, 3)), axis=0)
    coords = np.concatenate([np.zeros((len(coords), 1), np.int64), coords], 1).astype(np.int32)
    c = 6
    f = rng.standard_normal((len(coords), c))
    dw = rng.standard_normal((c, 3, 3, 3, c)) / 10
    db = rng.standard_normal(c)
    l0, b0 = rng.standard_normal((4 * c, c)), rng.standard_normal(4 * c)
    l2, b2 = rng.standard_normal((c, 4 * c)), rng.standard_normal(c)
    km = oracle.kmap_sorted(coords, (10, 10, 10))
    got = oracle.convnext_block(f, km, dw, db, l0, b0, l2, b2)
    h = torch.from_numpy(oracle.dense_conv3d_check(coords, f, dw, db, (10, 10, 10), 1))
    h = F.layer_norm(h, (c,), eps=1e-6)
    h = F.linear(h, torch.from_numpy(l0), torch.from_numpy(b0))
    h = F.silu(F.layer_norm(h, (4 * c,), eps=1e-6))
    h = F.linear(h, torch.from_numpy(l2), torch.from_numpy(b2)) + torch.from_numpy(f)
    np.testing.assert_allclose(got, h.numpy(), rtol=1e-9, atol=1e-9)


def test_subdivide_oracle_properties(oracle):
    rng = np.random.default_rng(23)
    coords = np.unique(rng.integers(0, 50, (400, 4)) * np.array([0, 1, 1, 1]) + np.array([1, 0, 0, 0]) *
                       rng.integers(0, 3, (400, 1)), axis=0).astype(np.int32)
    f = rng.standard_normal((len(coords), 3))
    fine, ff = oracle.subdivide2(coords, f)
    assert fine.shape == (8 * len(coords), 4)
    assert len(np.unique(fine, axis=0)) == len(fine)
    parents = np.concatenate([fine[:, :1], fine[:, 1:] >> 1], 1)
    assert np.array_equal(parents, np.repeat(coords, 8, axis=0))
    assert np.array_equal(ff, np.repeat(f, 8, axis=0))
    # down-sampling the children gives the voxels back, each with all 8 slots filled
    p, dmap = oracle.down2_map(fine)
    assert np.array_equal(p, coords[np.lexsort(coords.T[::-1])])
    assert np.all(dmap >= 0)
    mask = rng.random((len(coords), 8)) < 0.3
    fm, fmf = oracle.subdivide2(coords, f, mask)
    assert len(fm) == mask.sum()
    keep = mask.ravel()
    assert np.array_equal(fm, fine[keep]) and np.array_equal(fmf, ff[keep])


def test_attention_oracle_matches_torch_sdpa(oracle):
    import torch
    rng = np.random.default_rng(31)
    lq, lk = [5, 0, 17, 3], [7, 4, 0, 11]
    cq, ck = np.concatenate([[0], np.cumsum(lq)]), np.concatenate([[0], np.cumsum(lk)])
    q = rng.standard_normal((cq[-1], 3, 64))
    k = rng.standard_normal((ck[-1], 3, 64))
    v = rng.standard_normal((ck[-1], 3, 64))
    out = oracle.attention_varlen(q, k, v, cq, ck)
    for b in range(4):
        s, t = slice(cq[b], cq[b + 1]), slice(ck[b], ck[b + 1])
        if lq[b] == 0:
            continue
        if lk[b] == 0:
            assert not out[s].any()
            continue
        T = lambda x, sl: torch.from_numpy(x[sl]).transpose(0, 1)
        ref = torch.nn.functional.scaled_dot_product_attention(T(q, s), T(k, t), T(v, t)).transpose(0, 1).numpy()
        np.testing.assert_allclose(out[s], ref, rtol=1e-10, atol=1e-12)
