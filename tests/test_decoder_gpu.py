"""The decoder rows on the GPU: depthwise conv, ConvNeXt block, 2x2x2 subdivision.

Bounds: the depthwise conv within relative L2 1e-5 of the float64 oracle in
f32 and 5e-3 in bf16 / f16 (inputs rounded first, so the bound covers the
accumulation and the output rounding).  The ConvNeXt block chains a conv, two
LayerNorms, two GEMMs and a skip add; the oracle rounds to bf16 where the
engine stores bf16 and the bound is 5e-3 relative L2 (1e-4 in f32, where the
two GEMMs run as plain f32 cuBLAS GEMMs).  Subdivision is integer work:
coords, parents and copied feature rows bit-exact.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 5e-3, torch.float16: 5e-3}
BLOCK_TOL = {torch.float32: 1e-4, torch.bfloat16: 5e-3}


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _f64(t):
    return t.float().cpu().numpy().astype(np.float64)


def _coords(pkg, cuda, scale=0.3, cfg=2):
    w = pkg.workloads.make_workload(cfg, scale=scale)
    return w, torch.from_numpy(w.coords).to(cuda)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("c", [8, 64, 72, 200, 256])
def test_depthwise_conv_matches_oracle(pkg, oracle, cuda, dtype, c):
    w, coords = _coords(pkg, cuda)
    rng = np.random.default_rng(c)
    km = pkg.build_kmap(coords)
    f = torch.from_numpy(rng.standard_normal((w.n, c)).astype(np.float32)).to(cuda, dtype)
    W = torch.from_numpy((rng.standard_normal((c, 3, 3, 3, 1)) / np.sqrt(27)).astype(np.float32)).to(cuda, dtype)
    b = torch.from_numpy((0.1 * rng.standard_normal(c)).astype(np.float32)).to(cuda, dtype)
    out = pkg.conv3d_depthwise(km, f, W, b)
    ref = oracle.conv_depthwise(_f64(f), oracle.kmap_sorted(w.coords, w.spatial_shape), _f64(W), _f64(b))
    assert rel_l2(_f64(out), ref) < TOL[dtype]


def test_depthwise_conv_without_bias_and_dilated(pkg, oracle, cuda):
    w, coords = _coords(pkg, cuda)
    rng = np.random.default_rng(3)
    km = pkg.build_kmap(coords, dilation=(1, 2, 3))
    f = torch.from_numpy(rng.standard_normal((w.n, 32)).astype(np.float32)).to(cuda)
    W = torch.from_numpy(rng.standard_normal((32, 27)).astype(np.float32)).to(cuda)
    out = pkg.conv3d_depthwise(km, f, W)
    ref = oracle.conv_depthwise(_f64(f), oracle.kmap_sorted(w.coords, w.spatial_shape, dilation=(1, 2, 3)), _f64(W))
    assert rel_l2(_f64(out), ref) < 1e-5


def test_depthwise_conv_equals_dense_conv_with_diagonal_weight(pkg, cuda):
    """A (C, 3, 3, 3, 1) weight is the dense conv whose (C, v, C) slabs are
    diagonal; in f32 both paths sum the same products in the same order."""
    w, coords = _coords(pkg, cuda)
    rng = np.random.default_rng(4)
    km = pkg.build_kmap(coords)
    c = 16
    f = torch.from_numpy(rng.standard_normal((w.n, c)).astype(np.float32)).to(cuda)
    Wd = torch.from_numpy(rng.standard_normal((c, 27)).astype(np.float32)).to(cuda)
    dense = torch.zeros((c, 27, c), device=cuda)
    dense[torch.arange(c), :, torch.arange(c)] = Wd
    a = pkg.conv3d_depthwise(km, f, Wd)
    d = pkg.conv3d(km, f, dense.view(c, 3, 3, 3, c))
    assert torch.allclose(a, d, rtol=1e-5, atol=1e-5)


def test_depthwise_conv_refuses_bad_shapes(pkg, cuda):
    _, coords = _coords(pkg, cuda, scale=0.01)
    km = pkg.build_kmap(coords)
    f = torch.zeros((km.n_in, 12), device=cuda)
    with pytest.raises(pkg.SparseConvError, match="multiple of 8"):
        pkg.conv3d_depthwise(km, f, torch.zeros((12, 27), device=cuda))
    kd = pkg.build_down2(coords)
    with pytest.raises(ValueError):
        pkg.conv3d_depthwise(kd, torch.zeros((kd.n_in, 16), device=cuda), torch.zeros((16, 27), device=cuda))


def test_depthwise_conv_empty_map(pkg, cuda):
    km = pkg.build_kmap(torch.zeros((0, 4), dtype=torch.int32, device=cuda))
    out = pkg.conv3d_depthwise(km, torch.zeros((0, 16), device=cuda), torch.zeros((16, 27), device=cuda))
    assert out.shape == (0, 16)


def _block_weights(rng, c, depthwise, cuda, dtype):
    def t(shape, s):
        return torch.from_numpy((s * rng.standard_normal(shape)).astype(np.float32)).to(cuda, dtype)
    dw = t((c, 3, 3, 3, 1), 1 / np.sqrt(27)) if depthwise else t((c, 3, 3, 3, c), 1 / np.sqrt(27 * c))
    return dw, t(c, 0.1), t((4 * c, c), 1 / np.sqrt(c)), t(4 * c, 0.1), t((c, 4 * c), 1 / np.sqrt(4 * c)), t(c, 0.1)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("depthwise", [False, True])
@pytest.mark.parametrize("c", [64, 128])
def test_convnext_block_matches_oracle(pkg, oracle, cuda, dtype, depthwise, c):
    w, coords = _coords(pkg, cuda, scale=0.1)
    rng = np.random.default_rng(c + depthwise)
    f = torch.from_numpy(rng.standard_normal((w.n, c)).astype(np.float32)).to(cuda, dtype)
    ws = _block_weights(rng, c, depthwise, cuda, dtype)
    y = pkg.sparse_convnext_block(pkg.SparseTensor(f, coords), *ws)
    kmap = oracle.kmap_sorted(w.coords, w.spatial_shape)
    ref = oracle.convnext_block(_f64(f), kmap, *[_f64(t) for t in ws], round_to_bf16=dtype == torch.bfloat16)
    assert rel_l2(_f64(y.feats), ref) < BLOCK_TOL[dtype]


def test_convnext_block_linear_layouts_agree(pkg, cuda):
    """(in, out) matrices as the TS matmul takes them give the same block as
    torch.nn.Linear (out, in) weights."""
    _, coords = _coords(pkg, cuda)
    rng = np.random.default_rng(9)
    c = 64
    f = torch.from_numpy(rng.standard_normal((coords.shape[0], c)).astype(np.float32)).to(cuda)
    dw, db, l0, b0, l2, b2 = _block_weights(rng, c, True, cuda, torch.float32)
    x = pkg.SparseTensor(f, coords)
    a = pkg.sparse_convnext_block(x, dw, db, l0, b0, l2, b2)
    b = pkg.sparse_convnext_block(x, dw, db, l0.t().contiguous(), b0, l2.t().contiguous(), b2, linear_layout="in_out")
    assert torch.equal(a.feats, b.feats)


def test_convnext_block_without_conv(pkg, oracle, cuda):
    w, coords = _coords(pkg, cuda)
    rng = np.random.default_rng(10)
    c = 64
    f = torch.from_numpy(rng.standard_normal((w.n, c)).astype(np.float32)).to(cuda)
    _, _, l0, b0, l2, b2 = _block_weights(rng, c, True, cuda, torch.float32)
    y = pkg.sparse_convnext_block(pkg.SparseTensor(f, coords), None, None, l0, b0, l2, b2)
    ref = oracle.convnext_block(_f64(f), None, None, None, _f64(l0), _f64(b0), _f64(l2), _f64(b2))
    assert rel_l2(_f64(y.feats), ref) < 1e-4


@pytest.mark.parametrize("masked", ["none", "bool", "bits", "zero"])
def test_subdivide_matches_oracle(pkg, oracle, cuda, masked):
    w, coords = _coords(pkg, cuda, scale=0.5)
    rng = np.random.default_rng(11)
    f = torch.from_numpy(rng.standard_normal((w.n, 24)).astype(np.float32)).to(cuda, torch.bfloat16)
    mask_np = None
    mask = None
    if masked == "bool":
        mask_np = rng.random((w.n, 8)) < 0.4
        mask = torch.from_numpy(mask_np).to(cuda)
    elif masked == "bits":
        bits = rng.integers(0, 256, w.n).astype(np.uint8)
        mask_np = (bits[:, None] >> np.arange(8)[None] & 1).astype(bool)
        mask = torch.from_numpy(bits).to(cuda)
    elif masked == "zero":
        mask_np = np.zeros((w.n, 8), bool)
        mask = torch.from_numpy(mask_np).to(cuda)
    fine, parent = pkg.subdivide2(pkg.SparseTensor(f, coords), mask)
    ref_c, ref_f = oracle.subdivide2(w.coords, f.cpu().view(torch.int16).numpy(), mask_np)
    assert np.array_equal(fine.coords.cpu().numpy(), ref_c)
    assert np.array_equal(fine.feats.cpu().view(torch.int16).numpy(), ref_f)
    assert np.array_equal(coords[parent.long()].cpu().numpy()[:, 1:], ref_c[:, 1:] >> 1)
    assert fine.scale == (0.5, 0.5, 0.5)


def test_subdivide_down2_round_trip(pkg, oracle, cuda):
    """Subdividing and then down-sampling gives back the voxels (as unique
    sorted parents) and every child's down-sample slot is its child index."""
    w, coords = _coords(pkg, cuda, scale=0.02)
    f = torch.zeros((w.n, 8), device=cuda)
    fine, parent = pkg.subdivide2(pkg.SparseTensor(f, coords))
    kd = pkg.build_down2(fine.coords)
    p_ref, _ = oracle.down2_map(fine.coords.cpu().numpy())
    assert np.array_equal(kd.out_coords().cpu().numpy(), p_ref)
    order = np.lexsort(w.coords.T[::-1])
    assert np.array_equal(p_ref, w.coords[order])
    dmap = kd.export().cpu().numpy()
    # child s of original voxel p is fine row 8p + s and sits in slot s
    assert np.array_equal(dmap, 8 * order[:, None] + np.arange(8)[None, :])


def test_subdivided_tensor_conv(pkg, oracle, cuda):
    """A subm conv on the fine coords of a masked subdivision."""
    w, coords = _coords(pkg, cuda, scale=0.02)
    rng = np.random.default_rng(12)
    f = torch.from_numpy(rng.standard_normal((w.n, 32)).astype(np.float32)).to(cuda, torch.bfloat16)
    mask = torch.from_numpy(rng.random((w.n, 8)) < 0.5).to(cuda)
    fine, _ = pkg.subdivide2(pkg.SparseTensor(f, coords), mask)
    W = torch.from_numpy((rng.standard_normal((32, 3, 3, 3, 32)) / np.sqrt(27 * 32)).astype(np.float32)).to(
        cuda, torch.bfloat16)
    km = pkg.build_kmap(fine.coords)
    out = pkg.conv3d(km, fine.feats, W)
    fc = fine.coords.cpu().numpy()
    ref_map = oracle.kmap_sorted(fc, tuple(int(v) + 1 for v in fc[:, 1:].max(0)))
    assert np.array_equal(km.export().cpu().numpy(), ref_map)
    assert rel_l2(_f64(out), oracle.conv_gather(_f64(fine.feats), ref_map, _f64(W))) < 5e-3


def test_subdivide_full_c4_masked(pkg, oracle, cuda):
    """configs[3]'s 2.1M voxels (more than 1024 scan blocks) with a random
    child mask: coords, parents and feature rows bit-exact."""
    w = pkg.workloads.make_workload(4)
    coords = torch.from_numpy(w.coords).to(cuda)
    rng = np.random.default_rng(14)
    f16 = rng.integers(-32768, 32767, (w.n, 8)).astype(np.int16)
    f = torch.from_numpy(f16).to(cuda).view(torch.bfloat16)
    bits = rng.integers(0, 256, w.n).astype(np.uint8)
    fine, parent = pkg.subdivide2(pkg.SparseTensor(f, coords), torch.from_numpy(bits).to(cuda))
    mask_np = (bits[:, None] >> np.arange(8)[None] & 1).astype(bool)
    ref_c, ref_f = oracle.subdivide2(w.coords, f16, mask_np)
    assert np.array_equal(fine.coords.cpu().numpy(), ref_c)
    assert np.array_equal(fine.feats.view(torch.int16).cpu().numpy(), ref_f)
    assert np.array_equal(parent.cpu().numpy(), np.repeat(np.arange(w.n), mask_np.sum(1)))


def test_subdivide_empty_and_errors(pkg, cuda):
    x = pkg.SparseTensor(torch.zeros((0, 8), device=cuda), torch.zeros((0, 4), dtype=torch.int32, device=cuda))
    fine, parent = pkg.subdivide2(x)
    assert fine.coords.shape == (0, 4) and parent.shape == (0,)
    fine, _ = pkg.subdivide2(x, torch.zeros((0, 8), dtype=torch.bool, device=cuda))
    assert fine.feats.shape == (0, 8)
    y = pkg.SparseTensor(torch.zeros((4, 3), device=cuda), torch.zeros((4, 4), dtype=torch.int32, device=cuda))
    with pytest.raises(ValueError, match="16 bytes"):
        pkg.subdivide2(y)
    z = pkg.SparseTensor(torch.zeros((4, 4), device=cuda), torch.zeros((4, 4), dtype=torch.int32, device=cuda))
    with pytest.raises(ValueError):
        pkg.subdivide2(z, torch.zeros((4, 7), dtype=torch.bool, device=cuda))


def test_coords_cache_to_kmap(pkg, oracle, cuda, tmp_path):
    """A `.coords.bin` / `.attrs.bin` cache (3-column, as the mesh pipeline
    reads it) loads onto the device and builds the same map as the oracle."""
    w = pkg.workloads.make_workload(2, scale=0.05)
    assert np.all(w.coords[:, 0] == 0)                   # one shape: xyz rows are unique
    rng = np.random.default_rng(13)
    attrs = rng.random((w.n, 6)).astype(np.float32)
    prefix = str(tmp_path / "mesh.glb")
    pkg.coords_io.write_cache(prefix, w.coords[:, 1:], attrs)
    x = pkg.coords_io.load_sparse(prefix, device=cuda, pad_channels=8)
    assert x.feats.shape == (w.n, 8)
    assert torch.equal(x.feats[:, :6].cpu(), torch.from_numpy(attrs))
    km = pkg.build_kmap(x.coords)
    c4 = np.concatenate([np.zeros((w.n, 1), np.int32), w.coords[:, 1:]], 1)
    assert np.array_equal(km.export().cpu().numpy(), oracle.kmap_sorted(c4, w.spatial_shape))
    out = pkg.conv3d_depthwise(km, x.feats, torch.ones((8, 27), device=cuda))
    assert out.shape == (w.n, 8)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("c", [12, 16, 24, 64, 96, 200, 256, 1000, 4096])
@pytest.mark.parametrize("silu", [False, True])
def test_layernorm_silu_matches_torch(pkg, cuda, dtype, c, silu):
    """The engine's in-place row LayerNorm (no affine, eps 1e-6) + optional
    SiLU against torch in float64, over the vectorised widths and the scalar
    fallback (rows that are not a whole number of 16-byte vectors)."""
    rng = np.random.default_rng(c)
    n = 5003
    x = torch.from_numpy((3 * rng.standard_normal((n, c)) + 1).astype(np.float32)).to(cuda, dtype)
    ref = torch.nn.functional.layer_norm(x.double(), (c,), eps=1e-6)
    if silu:
        ref = torch.nn.functional.silu(ref)
    y = pkg.layernorm_silu(x.clone(), silu=silu)
    assert rel_l2(_f64(y), ref.cpu().numpy()) < TOL[dtype]
