"""Halo-staged conv (maps built with halo=True) against the default map and the oracle.

Both conv kernels accumulate chunk by chunk and offset by offset in the same
order, so a halo map must give results bit-identical to the default
(mask-sorted) map; the oracle check bounds both.  Tiles that gather more
distinct rows than a halo slot holds (416; shuffled row order) are gathered
straight from global memory by the same kernel.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _inputs(pkg, cuda, cfg, scale, ci, co, dtype=torch.bfloat16, seed=0):
    w = pkg.workloads.make_workload(cfg, scale=scale)
    rng = np.random.default_rng(seed)
    f = torch.from_numpy(rng.standard_normal((w.n, ci)).astype(np.float32)).to(cuda, dtype)
    W = torch.from_numpy((rng.standard_normal((co, 3, 3, 3, ci)) / np.sqrt(27 * ci)).astype(np.float32)).to(cuda, dtype)
    b = torch.from_numpy((0.1 * rng.standard_normal(co)).astype(np.float32)).to(cuda, dtype)
    return w, f, W, b


@pytest.mark.parametrize("ci,co", [(128, 128), (64, 64), (192, 96), (64, 16), (128, 48)])
def test_halo_conv_equals_default_map(pkg, oracle, cuda, ci, co):
    w, f, W, b = _inputs(pkg, cuda, 2, 0.3, ci, co)
    c = torch.from_numpy(w.coords).to(cuda)
    km_h = pkg.build_kmap(c, halo=True)
    km_d = pkg.build_kmap(c)
    info = km_h.info()
    assert 0 < info["halo_max"] <= 416
    assert km_d.info()["halo_max"] == -1
    assert torch.equal(km_h.export(), km_d.export())
    out_h = pkg.conv3d(km_h, f, W, b)
    out_d = pkg.conv3d(km_d, f, W, b)
    torch.cuda.synchronize()
    assert torch.equal(out_h, out_d)
    ref = oracle.conv_gather(f.float().cpu().numpy(), km_d.export().cpu().numpy(), W.float().cpu().numpy(),
                             b.float().cpu().numpy())
    assert rel_l2(out_h.float().cpu().numpy(), ref) < 5e-3


def test_halo_conv_f16_and_epilogues(pkg, cuda):
    ci = co = 128
    w, f, W, b = _inputs(pkg, cuda, 3, 0.35, ci, co, dtype=torch.float16, seed=1)
    c = torch.from_numpy(w.coords).to(cuda)
    km_h = pkg.build_kmap(c, halo=True)
    km_d = pkg.build_kmap(c)
    res = torch.randn_like(f)
    for kw in ({"silu": True}, {"layernorm": True, "silu": True}, {"residual": res}):
        out_h = pkg.conv3d(km_h, f, W, b, **kw)
        out_d = pkg.conv3d(km_d, f, W, b, **kw)
        torch.cuda.synchronize()
        assert torch.equal(out_h, out_d), kw


def test_halo_overflow_gathers_directly(pkg, oracle, cuda):
    # shuffled rows: a tile's 128 outputs are scattered, so its halo exceeds the
    # 416-row slot and the conv gathers those tiles' rows from global memory
    ci = co = 64
    w, f, W, b = _inputs(pkg, cuda, 2, 0.3, ci, co, seed=2)
    perm = pkg.workloads.shuffle_rows(w.n, 5)
    coords = np.ascontiguousarray(w.coords[perm])
    c = torch.from_numpy(coords).to(cuda)
    km_h = pkg.build_kmap(c, halo=True)
    assert km_h.info()["halo_max"] > 416
    fs = f.index_select(0, torch.from_numpy(perm).to(cuda))
    out = pkg.conv3d(km_h, fs, W, b)
    assert torch.equal(out, pkg.conv3d(pkg.build_kmap(c), fs, W, b))
    ref = oracle.conv_gather(fs.float().cpu().numpy(), oracle.kmap_sorted(coords, w.spatial_shape),
                             W.float().cpu().numpy(), b.float().cpu().numpy())
    assert rel_l2(out.float().cpu().numpy(), ref) < 5e-3


def test_halo_full_c2(pkg, oracle, cuda):
    w = pkg.workloads.make_workload(2)
    c = torch.from_numpy(w.coords).to(cuda)
    f = torch.from_numpy(w.feats).to(cuda, torch.bfloat16)
    W = torch.from_numpy(w.weight).to(cuda, torch.bfloat16)
    km_h = pkg.build_kmap(c, halo=True)
    km_d = pkg.build_kmap(c)
    assert km_h.info()["halo_max"] <= 416
    out_h = pkg.conv3d(km_h, f, W)
    out_d = pkg.conv3d(km_d, f, W)
    torch.cuda.synchronize()
    assert torch.equal(out_h, out_d)
    pkg.get_engine(cuda).synchronize()
