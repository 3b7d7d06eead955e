"""Full-size parity on the GPU: the BASELINE configurations at their full sizes.

Bounds as in the other parity tests: maps bit-exact; bf16 convs within
relative L2 5e-3 of the float64 oracle.  Where the engine stores an
intermediate in bf16 (the ResBlock's hidden activation, the activations
between the chained down / subm / up convs) the oracle rounds it to bf16 the
same way, so the bound covers the accumulation and the output rounding.  The
1024^3 and 512^3 convs are checked on seeded samples of output rows: the oracle
computes only those rows (its neighbour lookups still search every voxel).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

BF16_TOL = 5e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _f64(t):
    return t.float().cpu().numpy().astype(np.float64)


def _conv_rows(oracle, feats, kmap_rows, weight64):
    """Oracle conv of the given map rows, reading only the input rows they use
    (``feats``: a tensor; keeps the float64 copy small at full size)."""
    km = np.asarray(kmap_rows)
    used = np.unique(km[km >= 0])
    pos = np.full(int(feats.shape[0]), -1, np.int64)
    pos[used] = np.arange(len(used))
    compact = _f64(feats.index_select(0, torch.from_numpy(used).to(feats.device)))
    remapped = np.where(km >= 0, pos[np.maximum(km, 0)], -1)
    return oracle.conv_gather(compact, remapped, weight64)


def _rows(t, idx):
    return t.index_select(0, torch.from_numpy(np.asarray(idx)).to(t.device))


def test_c3_full_resblock(pkg, oracle, cuda):
    """configs[2] at full size: 4 shapes, 256 channels, conv -> LN -> SiLU -> conv + skip."""
    w = pkg.workloads.make_workload(3)
    c = torch.from_numpy(w.coords).to(cuda)
    f = torch.from_numpy(w.feats).to(cuda, torch.bfloat16)
    w1 = torch.from_numpy(w.weight).to(cuda, torch.bfloat16)
    w2 = torch.from_numpy(w.extra["weight2"]).to(cuda, torch.bfloat16)
    y = pkg.sparse_resblock(pkg.SparseTensor(f, c), w1, None, w2, None)
    km = pkg.build_kmap(c)
    h = pkg.conv3d(km, f, w1, silu=True, layernorm=True)
    ref_map = oracle.kmap_sorted(w.coords, w.spatial_shape)
    assert np.array_equal(km.export().cpu().numpy(), ref_map)
    f64, w1_64, w2_64 = _f64(f), _f64(w1), _f64(w2)
    h_ref = oracle.silu(oracle.layer_norm(oracle.conv_gather(f64, ref_map, w1_64)))
    assert rel_l2(_f64(h), h_ref) < BF16_TOL
    out_ref = oracle.resblock(f64, ref_map, w1_64, None, w2_64, None, hidden_bf16=True)
    assert rel_l2(_f64(y.feats), out_ref) < BF16_TOL


def test_c4_full_down_subm_up_chain(pkg, oracle, cuda):
    """configs[3] at full size (2.1M voxels): every map bit-exact, every conv on
    50k sampled rows fed the engine's own input, and the whole chain on 1,000
    sampled output rows from the inputs alone, intermediates rounded to bf16."""
    w = pkg.workloads.make_workload(4)
    rng = np.random.default_rng(44)
    c = torch.from_numpy(w.coords).to(cuda)
    f = torch.from_numpy(w.feats).to(cuda, torch.bfloat16)
    wd = torch.from_numpy(w.weight).to(cuda, torch.bfloat16)
    ws = torch.from_numpy(w.extra["w_sub"]).to(cuda, torch.bfloat16)
    wu = torch.from_numpy(w.extra["w_up"]).to(cuda, torch.bfloat16)
    kd = pkg.build_down2(c)
    parents = kd.out_coords()
    ks = pkg.build_kmap(parents)
    ku = pkg.build_up2(kd)
    hd = pkg.conv3d(kd, f, wd)
    hs = pkg.conv3d(ks, hd, ws)
    out = pkg.conv3d(ku, hs, wu)
    # maps
    p_ref, dmap = oracle.down2_map(w.coords)
    assert np.array_equal(parents.cpu().numpy(), p_ref)
    assert np.array_equal(kd.export().cpu().numpy(), dmap)
    umap = oracle.up2_map(w.coords, p_ref)
    assert np.array_equal(ku.export().cpu().numpy(), umap)
    smap = oracle.kmap_sorted(p_ref, tuple(s // 2 for s in w.spatial_shape))
    assert np.array_equal(ks.export().cpu().numpy(), smap)
    # each conv on sampled rows, fed the engine's own input
    wd64, ws64, wu64 = _f64(wd), _f64(ws), _f64(wu)
    sp = rng.choice(len(p_ref), 50000, replace=False)
    sf = rng.choice(w.n, 50000, replace=False)
    assert rel_l2(_f64(_rows(hd, sp)), _conv_rows(oracle, f, dmap[sp], wd64)) < BF16_TOL
    assert rel_l2(_f64(_rows(hs, sp)), _conv_rows(oracle, hd, smap[sp], ws64)) < BF16_TOL
    assert rel_l2(_f64(_rows(out, sf)), _conv_rows(oracle, hs, umap[sf], wu64)) < BF16_TOL
    # the whole chain on a few output rows
    rows = rng.choice(w.n, 1000, replace=False)
    par = umap[rows].max(1)                      # parent of each sampled fine row
    up = np.unique(par)
    need = np.unique(smap[up].ravel())           # parents its subm conv reads
    need = need[need >= 0]
    hd_c = oracle.round_bf16(_conv_rows(oracle, f, dmap[need], wd64))
    pos = np.full(len(p_ref), -1, np.int64)
    pos[need] = np.arange(len(need))
    hs_c = oracle.round_bf16(oracle.conv_gather(hd_c, np.where(smap[up] >= 0, pos[np.maximum(smap[up], 0)], -1),
                                                ws64))
    posu = np.full(len(p_ref), -1, np.int64)
    posu[up] = np.arange(len(up))
    um = umap[rows]
    out_ref = oracle.conv_gather(hs_c, np.where(um >= 0, posu[np.maximum(um, 0)], -1), wu64)
    assert rel_l2(_f64(_rows(out, rows)), out_ref) < BF16_TOL


def test_c5_full_conv_sampled(pkg, oracle, cuda):
    """configs[4] at full size (6.1M voxels, 32 channels): 200k sampled output rows."""
    w = pkg.workloads.make_workload(5)
    c = torch.from_numpy(w.coords).to(cuda)
    f = torch.from_numpy(w.feats).to(cuda, torch.bfloat16)
    W = torch.from_numpy(w.weight).to(cuda, torch.bfloat16)
    out = pkg.conv3d(pkg.build_kmap(c), f, W)
    rows = np.random.default_rng(55).choice(w.n, 200000, replace=False)
    km_rows = oracle.kmap_sorted(w.coords, w.spatial_shape, rows=rows)
    ref = _conv_rows(oracle, f, km_rows, _f64(W))
    assert rel_l2(_f64(_rows(out, rows)), ref) < BF16_TOL
    pkg.get_engine(cuda).synchronize()
