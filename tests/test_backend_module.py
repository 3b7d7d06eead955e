"""The SPARSE_CONV_BACKEND=b200 module (conv_b200.py) as the reference's
backend dispatcher would load it: selection by the environment variable,
module construction in the checkpoint weight layout, and the refusal of CPU
inputs (there is no CPU path).  The GPU test checks its forward against the
direct conv3d calls."""
import numpy as np
import pytest
import torch


def test_backend_selected_by_environment(pkg, monkeypatch):
    monkeypatch.setenv("SPARSE_CONV_BACKEND", "b200")
    mod = pkg.conv_b200.load_backend()
    assert mod is pkg.conv_b200 and mod.BACKEND_NAME == "b200"
    monkeypatch.setenv("SPARSE_CONV_BACKEND", "none")
    with pytest.raises(ValueError):
        pkg.conv_b200.load_backend()


def test_modules_hold_the_checkpoint_layout(pkg):
    m = pkg.conv_b200.SparseConv3d(16, 32, 3)
    assert tuple(m.weight.shape) == (32, 3, 3, 3, 16) and tuple(m.bias.shape) == (32,)
    assert m.cache_key() == "conv_neighbors_3x3x3_dil1x1x1"
    d = pkg.conv_b200.SparseConv3d(16, 32, 2, stride=2, bias=False)
    assert tuple(d.weight.shape) == (32, 2, 2, 2, 16) and d.bias is None
    u = pkg.conv_b200.SparseInverseConv3d(32, 16)
    assert tuple(u.weight.shape) == (16, 2, 2, 2, 32)
    with pytest.raises(NotImplementedError):
        pkg.conv_b200.SparseConv3d(16, 16, 5)
    with pytest.raises(NotImplementedError):
        pkg.conv_b200.SparseConv3d(16, 16, 3, stride=3)


def test_cpu_input_is_refused(pkg):
    m = pkg.conv_b200.SparseConv3d(8, 8, 3)
    x = pkg.SparseTensor(torch.zeros((4, 8)), torch.zeros((4, 4), dtype=torch.int32))
    with pytest.raises(ValueError):
        m(x)


@pytest.mark.gpu
def test_backend_forward_matches_conv3d(pkg, cuda):
    w = pkg.workloads.make_workload(4, scale=0.15)
    c = torch.from_numpy(w.coords).to(cuda)
    rng = np.random.default_rng(21)
    f = torch.from_numpy(rng.standard_normal((w.n, 64)).astype(np.float32)).to(cuda, torch.bfloat16)
    B = pkg.conv_b200
    down = B.SparseConv3d(64, 128, 2, stride=2).to(cuda)
    subm = B.SparseConv3d(128, 128, 3).to(cuda)
    up = B.SparseInverseConv3d(128, 64).to(cuda)
    with torch.no_grad():
        for m in (down, subm, up):
            if m.bias is not None:
                m.bias.normal_(0, 0.1)
        x = pkg.SparseTensor(f, c)
        y = up(subm(down(x)))
        kd = pkg.build_down2(c)
        ks = pkg.build_kmap(kd.out_coords())
        ku = pkg.build_up2(kd)
        bf = lambda t: t.to(torch.bfloat16)
        hd = pkg.conv3d(kd, f, bf(down.weight), bf(down.bias))
        hs = pkg.conv3d(ks, hd, bf(subm.weight), bf(subm.bias))
        ref = pkg.conv3d(ku, hs, bf(up.weight), bf(up.bias))
    assert torch.equal(y.feats, ref)
    assert y.coords is c
