"""The allocation-free map build (sc_kmap_build_noalloc), called through the C ABI.

This entry point serves callers that must not let the library allocate device
memory (a host runtime that budgets all device memory itself, or a
latency-sensitive path that cannot wait on an allocator).  It must return the
same map as the regular build, call after call, since every call reuses the
same fixed scratch array; and it must refuse inputs above its fixed limit.
The file sorts last so that, if it fails, every other test has already run.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(pkg, eng, coords, dilation=1):
    n = coords.shape[0]
    out = torch.full((n, 27), -7, dtype=torch.int32, device=coords.device)
    eng.bind_stream()
    st = pkg._lib.lib().sc_kmap_build_noalloc(eng.handle, ctypes.c_void_p(coords.data_ptr()), n, dilation,
                                              ctypes.c_void_p(out.data_ptr()))
    return st, out


@pytest.mark.parametrize("cfg,scale,dil", [(1, 1.0, 1), (3, 0.35, 1), (1, 0.7, 2)])
def test_noalloc_matches_regular_build_on_repeated_calls(pkg, cuda, cfg, scale, dil):
    w = pkg.workloads.make_workload(cfg, scale=scale)
    perm = pkg.workloads.shuffle_rows(w.n, cfg)
    coords = torch.from_numpy(np.ascontiguousarray(w.coords[perm])).to(cuda)
    eng = pkg.get_engine(cuda)
    expected = pkg.build_kmap(coords, dilation=dil, engine=eng).export()
    for _ in range(2):  # the second call sees the first call's leftovers in the scratch
        st, got = _noalloc(pkg, eng, coords, dil)
        assert st == pkg._lib.SC_OK, pkg._lib.lib().sc_last_error(eng.handle)
        torch.cuda.synchronize()
        assert torch.equal(got, expected)  # integer map: bit-exact


def test_noalloc_alternating_inputs(pkg, cuda):
    eng = pkg.get_engine(cuda)
    a = torch.from_numpy(pkg.workloads.make_workload(1).coords).to(cuda)
    b = torch.from_numpy(pkg.workloads.make_workload(1, scale=0.5).coords).to(cuda)
    ea, eb = pkg.build_kmap(a, engine=eng).export(), pkg.build_kmap(b, engine=eng).export()
    for coords, exp in ((a, ea), (b, eb), (a, ea)):
        st, got = _noalloc(pkg, eng, coords)
        assert st == pkg._lib.SC_OK
        assert torch.equal(got, exp)


def test_noalloc_rejects_inputs_above_the_limit(pkg, cuda):
    eng = pkg.get_engine(cuda)
    n = pkg._lib.SC_NOALLOC_MAX_VOXELS + 1
    coords = torch.zeros((n, 4), dtype=torch.int32, device=cuda)
    st, _ = _noalloc(pkg, eng, coords)
    assert st == pkg._lib.SC_EINVAL
    assert b"131072" in pkg._lib.lib().sc_last_error(eng.handle)


def test_noalloc_reports_duplicates(pkg, cuda):
    eng = pkg.get_engine(cuda)
    w = pkg.workloads.make_workload(1, scale=0.5)
    c = np.concatenate([w.coords, w.coords[:1]], 0)
    st, _ = _noalloc(pkg, eng, torch.from_numpy(c).to(cuda))
    assert st == pkg._lib.SC_EDUP_COORD
    st, got = _noalloc(pkg, eng, torch.from_numpy(w.coords).to(cuda))  # usable afterwards
    assert st == pkg._lib.SC_OK
    assert torch.equal(got, pkg.build_kmap(torch.from_numpy(w.coords).to(cuda), engine=eng).export())
