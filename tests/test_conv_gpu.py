"""Conv parity on the GPU against the float64 CPU oracle.

Tolerances (relative L2 over the whole output): 1e-5 for the f32 path,
5e-3 for bf16 (inputs are rounded to bf16 first, so the bound covers only the
accumulation and the bf16 rounding of the output), 2e-3 for f16.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 5e-3, torch.float16: 2e-3}


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _setup(pkg, oracle, cuda, cfg, scale, ci, co, dtype, seed=0, K=27):
    w = pkg.workloads.make_workload(cfg, scale=scale)
    rng = np.random.default_rng(seed)
    f = torch.from_numpy(rng.standard_normal((w.n, ci)).astype(np.float32)).to(cuda, dtype)
    shape = (co, 3, 3, 3, ci) if K == 27 else (co, 2, 2, 2, ci)
    W = torch.from_numpy((rng.standard_normal(shape) / np.sqrt(K * ci)).astype(np.float32)).to(cuda, dtype)
    b = torch.from_numpy((0.1 * rng.standard_normal(co)).astype(np.float32)).to(cuda, dtype)
    return w, f, W, b


def test_c1_f32_matches_oracle(pkg, oracle, cuda):
    w = pkg.workloads.make_workload(1)
    c = torch.from_numpy(w.coords).to(cuda)
    km = pkg.build_kmap(c)
    f = torch.from_numpy(w.feats).to(cuda)
    W = torch.from_numpy(w.weight).to(cuda)
    b = torch.from_numpy(w.bias).to(cuda)
    out = pkg.conv3d(km, f, W, b).cpu().numpy()
    ref = oracle.conv_gather(w.feats, oracle.kmap_sorted(w.coords, w.spatial_shape), w.weight, w.bias)
    assert rel_l2(out, ref) < 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("ci,co", [(64, 64), (128, 128), (32, 32), (16, 48), (48, 16), (256, 256), (64, 384),
                                   (96, 160)])
def test_tc_conv_channels(pkg, oracle, cuda, dtype, ci, co):
    w, f, W, b = _setup(pkg, oracle, cuda, 2, 0.2, ci, co, dtype)
    km = pkg.build_kmap(torch.from_numpy(w.coords).to(cuda))
    out = pkg.conv3d(km, f, W, b).float().cpu().numpy()
    ref = oracle.conv_gather(f.float().cpu().numpy(), km.export().cpu().numpy(), W.float().cpu().numpy(),
                             b.float().cpu().numpy())
    assert rel_l2(out, ref) < TOL[dtype]


def test_c2_full_bf16(pkg, oracle, cuda):
    w = pkg.workloads.make_workload(2)
    c = torch.from_numpy(w.coords).to(cuda)
    km = pkg.build_kmap(c)
    f = torch.from_numpy(w.feats).to(cuda, torch.bfloat16)
    W = torch.from_numpy(w.weight).to(cuda, torch.bfloat16)
    out = pkg.conv3d(km, f, W).float().cpu().numpy()
    ref = oracle.conv_gather(f.float().cpu().numpy(), oracle.kmap_sorted(w.coords, w.spatial_shape),
                             W.float().cpu().numpy())
    assert rel_l2(out, ref) < 5e-3


@pytest.mark.parametrize("tile_sort", [True, False])
def test_tile_order_gives_same_result(pkg, cuda, tile_sort):
    w = pkg.workloads.make_workload(3, scale=0.4)
    c = torch.from_numpy(w.coords).to(cuda)
    f = torch.randn(w.n, 64, device=cuda, dtype=torch.bfloat16)
    W = torch.randn(64, 3, 3, 3, 64, device=cuda, dtype=torch.bfloat16) / 40
    a = pkg.conv3d(pkg.build_kmap(c, tile_sort=tile_sort), f, W)
    b = pkg.conv3d(pkg.build_kmap(c, tile_sort=True), f, W)
    # every output row is a fixed-order sum over its own offsets: identical bits
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_epilogues(pkg, oracle, cuda, dtype):
    w, f, W, b = _setup(pkg, oracle, cuda, 3, 0.3, 64, 64, dtype)
    km = pkg.build_kmap(torch.from_numpy(w.coords).to(cuda))
    kmn = km.export().cpu().numpy()
    base = oracle.conv_gather(f.float().cpu().numpy(), kmn, W.float().cpu().numpy(), b.float().cpu().numpy())
    res = torch.randn(w.n, 64, device=cuda).to(dtype)
    tol = TOL[dtype] * (4 if dtype == torch.float32 else 1)
    out = pkg.conv3d(km, f, W, b, silu=True).float().cpu().numpy()
    assert rel_l2(out, oracle.silu(base)) < tol
    out = pkg.conv3d(km, f, W, b, residual=res).float().cpu().numpy()
    assert rel_l2(out, base + res.float().cpu().numpy()) < tol
    out = pkg.conv3d(km, f, W, b, layernorm=True, silu=True, residual=res).float().cpu().numpy()
    exp = oracle.silu(oracle.layer_norm(base)) + res.float().cpu().numpy()
    assert rel_l2(out, exp) < tol * 2


def test_resblock_c3(pkg, oracle, cuda):
    w = pkg.workloads.make_workload(3, scale=0.5)
    c = torch.from_numpy(w.coords).to(cuda)
    ch = 256
    f = torch.from_numpy(w.feats).to(cuda, torch.bfloat16)
    w1 = torch.from_numpy(w.weight).to(cuda, torch.bfloat16)
    w2 = torch.from_numpy(w.extra["weight2"]).to(cuda, torch.bfloat16)
    x = pkg.SparseTensor(f, c)
    y = pkg.sparse_resblock(x, w1, None, w2, None)
    km = oracle.kmap_sorted(w.coords, w.spatial_shape)
    ref = oracle.resblock(f.float().cpu().numpy(), km, w1.float().cpu().numpy(), None, w2.float().cpu().numpy(), None)
    assert y.feats.shape == (w.n, ch)
    assert rel_l2(y.feats.float().cpu().numpy(), ref) < 1e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_down_up_conv(pkg, oracle, cuda, dtype):
    w = pkg.workloads.make_workload(4, scale=0.2)
    rng = np.random.default_rng(4)
    c = torch.from_numpy(w.coords).to(cuda)
    f = torch.from_numpy(rng.standard_normal((w.n, 64)).astype(np.float32)).to(cuda, dtype)
    wd = torch.from_numpy((rng.standard_normal((128, 2, 2, 2, 64)) / 23).astype(np.float32)).to(cuda, dtype)
    wu = torch.from_numpy((rng.standard_normal((64, 2, 2, 2, 128)) / 32).astype(np.float32)).to(cuda, dtype)
    bd = torch.from_numpy((0.1 * rng.standard_normal(128)).astype(np.float32)).to(cuda, dtype)
    x = pkg.SparseTensor(f, c)
    down = pkg.SparseConvDown2(wd, bd)(x)
    pc, dmap = oracle.down2_map(w.coords)
    assert np.array_equal(down.coords.cpu().numpy(), pc)
    exp_d = oracle.conv_gather(f.float().cpu().numpy(), dmap, wd.float().cpu().numpy(), bd.float().cpu().numpy())
    assert rel_l2(down.feats.float().cpu().numpy(), exp_d) < TOL[dtype]
    up = pkg.SparseConvUp2(wu)(down)
    assert up.coords is c
    exp_u = oracle.conv_gather(down.feats.float().cpu().numpy(), oracle.up2_map(w.coords, pc),
                               wu.float().cpu().numpy())
    assert rel_l2(up.feats.float().cpu().numpy(), exp_u) < TOL[dtype]


def test_conv_is_deterministic_and_leaves_padding(pkg, cuda):
    w = pkg.workloads.make_workload(2, scale=0.25)
    c = torch.from_numpy(w.coords).to(cuda)
    km = pkg.build_kmap(c)
    f = torch.randn(w.n, 128, device=cuda, dtype=torch.bfloat16)
    W = torch.randn(128, 3, 3, 3, 128, device=cuda, dtype=torch.bfloat16) / 60
    canary = torch.full((w.n + 256, 128), 7.0, device=cuda, dtype=torch.bfloat16)
    out1 = pkg.conv3d(km, f, W, out=canary[128:128 + w.n])
    out2 = pkg.conv3d(km, f, W)
    torch.cuda.synchronize()
    assert torch.equal(out1, out2)
    assert (canary[:128] == 7.0).all() and (canary[128 + w.n:] == 7.0).all()


def test_sparse_conv3d_module_caches_map(pkg, oracle, cuda):
    w = pkg.workloads.make_workload(1, scale=0.6)
    c = torch.from_numpy(w.coords).to(cuda)
    f = torch.from_numpy(w.feats).to(cuda)
    conv = pkg.SparseConv3d(torch.from_numpy(w.weight).to(cuda), torch.from_numpy(w.bias).to(cuda))
    x = pkg.SparseTensor(f, c)
    y = conv(x)
    km = x.get_spatial_cache(conv.cache_key())
    assert km is not None and y.get_spatial_cache(conv.cache_key()) is km
    z = conv(y.replace(f))
    assert torch.equal(y.feats, z.feats)
    out, km2 = pkg.sparse_conv3d_forward(f, c, conv.weight, conv.bias)
    assert torch.equal(out, y.feats)
    assert torch.equal(km2.export(), km.export())  # the functional path builds the same map


def test_dense_conv_invariant_on_gpu(pkg, oracle, cuda):
    # the reference's own check: sparse conv == dense F.conv3d at active voxels
    w = pkg.workloads.make_workload(1, scale=0.5)
    rng = np.random.default_rng(7)
    f = rng.standard_normal((w.n, 16)).astype(np.float32)
    W = (rng.standard_normal((16, 3, 3, 3, 16)) / 20).astype(np.float32)
    b = (0.1 * rng.standard_normal(16)).astype(np.float32)
    km = pkg.build_kmap(torch.from_numpy(w.coords).to(cuda))
    out = pkg.conv3d(km, torch.from_numpy(f).to(cuda), torch.from_numpy(W).to(cuda), torch.from_numpy(b).to(cuda))
    dense = oracle.dense_conv3d_check(w.coords, f, W, b, w.spatial_shape, 1)
    assert rel_l2(out.cpu().numpy(), dense) < 1e-5


def test_bad_arguments_raise(pkg, cuda):
    w = pkg.workloads.make_workload(1, scale=0.5)
    km = pkg.build_kmap(torch.from_numpy(w.coords).to(cuda))
    f = torch.randn(w.n, 40, device=cuda, dtype=torch.bfloat16)
    W = torch.randn(40, 3, 3, 3, 40, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(pkg.SparseConvError):
        pkg.conv3d(km, f, W)  # Ci not a multiple of 16 on the tensor-core path
    with pytest.raises(ValueError):
        pkg.conv3d(km, f[:-1], W)


def test_large_map_tile_order_matches_unsorted_tiles(pkg, oracle, cuda):
    # 2.2M outputs: every output row sums its offsets in the same order whatever
    # tile it lands in, so the mask-sorted map gives a bit-identical result to
    # the unsorted-tile map; a sample of rows is checked against the oracle.
    w = pkg.workloads.make_workload(5, scale=0.6)
    assert w.n > (1 << 20)
    c = torch.from_numpy(w.coords).to(cuda)
    km = pkg.build_kmap(c)
    km_plain = pkg.build_kmap(c, tile_sort=False)
    assert km.info()["num_pairs"] == km_plain.info()["num_pairs"]
    f = torch.from_numpy(w.feats).to(cuda, torch.bfloat16)
    W = torch.from_numpy(w.weight).to(cuda, torch.bfloat16)
    out = pkg.conv3d(km, f, W)
    ref = pkg.conv3d(km_plain, f, W)
    assert torch.equal(out, ref)
    sample = np.random.default_rng(0).choice(w.n, 20000, replace=False)
    full = oracle.kmap_sorted(w.coords, w.spatial_shape)
    got = km.export().cpu().numpy()
    assert np.array_equal(got[sample], full[sample])
    part = oracle.conv_gather(f.float().cpu().numpy(), full[sample], W.float().cpu().numpy())
    assert rel_l2(out.float().cpu().numpy()[sample], part) < TOL[torch.bfloat16]


def test_conv_cta_limit_gives_same_result(pkg, cuda):
    # fewer persistent CTAs (sc_set_conv_ctas) change the schedule, not the sums
    w = pkg.workloads.make_workload(2, scale=0.3)
    c = torch.from_numpy(w.coords).to(cuda)
    km = pkg.build_kmap(c)
    f = torch.from_numpy(w.feats).to(cuda, torch.bfloat16)
    W = torch.from_numpy(w.weight).to(cuda, torch.bfloat16)
    eng = pkg.get_engine(cuda)
    ref = pkg.conv3d(km, f, W)
    try:
        for ctas in (7, 64):
            eng.set_conv_ctas(ctas)
            assert torch.equal(pkg.conv3d(km, f, W), ref)
    finally:
        eng.set_conv_ctas(0)


@pytest.mark.parametrize("ci,co", [(256, 256), (128, 128), (32, 32)])
def test_map_built_on_one_stream_used_on_another(pkg, cuda, ci, co):
    """A map is complete when its build's stream work is: its work orders
    (one per tiles-per-item choice, used by convs with Co > 128, Co <= 128 and
    Ci = Co = 32) are written by the build itself, so a conv on a second
    stream that waits only for the build matches a conv on the first."""
    w = pkg.workloads.make_workload(2, scale=0.2)
    rng = np.random.default_rng(ci)
    c = torch.from_numpy(w.coords).to(cuda)
    f = torch.from_numpy(rng.standard_normal((w.n, ci)).astype(np.float32)).to(cuda, torch.bfloat16)
    W = torch.from_numpy((rng.standard_normal((co, 3, 3, 3, ci)) / np.sqrt(27 * ci)).astype(np.float32)).to(
        cuda, torch.bfloat16)
    ref = pkg.conv3d(pkg.build_kmap(c), f, W)
    sa, sb = torch.cuda.Stream(), torch.cuda.Stream()
    sa.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(sa):
        km = pkg.build_kmap(c, check=False)
    sb.wait_stream(sa)
    with torch.cuda.stream(sb):
        out = pkg.conv3d(km, f, W)
    torch.cuda.current_stream().wait_stream(sb)
    torch.cuda.synchronize()
    km.check()
    assert torch.equal(out, ref)
