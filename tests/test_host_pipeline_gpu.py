"""HostConvPipeline: host-to-host convs with overlapped transfers equal the device API."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(pkg, scale, seed, ci):
    w = pkg.workloads.make_workload(2, scale=scale, seed=seed)
    feats = np.random.default_rng(seed).standard_normal((w.n, ci)).astype(np.float32)
    return w.coords, feats


def test_pipeline_matches_device_api(pkg, cuda):
    ci, co = 64, 96
    rng = np.random.default_rng(0)
    W = torch.from_numpy((rng.standard_normal((co, 3, 3, 3, ci)) / np.sqrt(27 * ci)).astype(np.float32))
    W = W.to(cuda, torch.bfloat16)
    b = torch.from_numpy((0.1 * rng.standard_normal(co)).astype(np.float32)).to(cuda, torch.bfloat16)
    pipe = pkg.HostConvPipeline(W, b, depth=2)
    calls = []
    for k, scale in enumerate([0.2, 0.35, 0.1, 0.3, 0.25]):  # ragged sizes, slots reused and regrown
        coords, feats = _inputs(pkg, scale, 10 + k, ci)
        c_h = torch.from_numpy(coords).pin_memory()
        f_h = torch.from_numpy(feats).to(torch.bfloat16).pin_memory()
        o_h = torch.empty((len(coords), co), dtype=torch.bfloat16).pin_memory()
        pipe.submit(c_h, f_h, o_h)
        calls.append((c_h, f_h, o_h))
    pipe.synchronize()
    for c_h, f_h, o_h in calls:
        ref = pkg.conv3d(pkg.build_kmap(c_h.to(cuda)), f_h.to(cuda), W, b).cpu()
        assert torch.equal(o_h, ref)


def test_pipeline_reports_duplicate_coords(pkg, cuda):
    coords, feats = _inputs(pkg, 0.1, 3, 16)
    coords = np.concatenate([coords, coords[:1]], 0)
    feats = np.concatenate([feats, feats[:1]], 0)
    W = torch.zeros((16, 3, 3, 3, 16), dtype=torch.bfloat16, device=cuda)
    pipe = pkg.HostConvPipeline(W)
    c_h = torch.from_numpy(coords).pin_memory()
    f_h = torch.from_numpy(feats).to(torch.bfloat16).pin_memory()
    o_h = torch.empty((len(coords), 16), dtype=torch.bfloat16).pin_memory()
    pipe.submit(c_h, f_h, o_h)
    with pytest.raises(pkg.DuplicateCoordError):
        pipe.synchronize()


def test_pipeline_rejects_device_tensors(pkg, cuda):
    W = torch.zeros((16, 3, 3, 3, 16), dtype=torch.bfloat16, device=cuda)
    pipe = pkg.HostConvPipeline(W)
    c = torch.zeros((4, 4), dtype=torch.int32, device=cuda)
    with pytest.raises(ValueError):
        pipe.submit(c, torch.zeros((4, 16), dtype=torch.bfloat16), torch.zeros((4, 16), dtype=torch.bfloat16))
