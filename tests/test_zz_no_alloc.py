"""The allocation-free map build (sc_kmap_build_noalloc), called through the C ABI.

This entry point serves callers that must not let the library allocate device
memory (a host runtime that budgets all device memory itself, or a
latency-sensitive path that cannot wait on an allocator).  It must return the
same map as the regular build, call after call, since every call reuses the
same fixed scratch array; it must refuse inputs above its fixed limit; and it
must leave the device's free memory, the library's memory pool and torch's
allocator exactly as they were.
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


def _pool_used(device_index):
    """Bytes in use in the device's default memory pool (the library's allocator)."""
    from cuda.bindings import runtime as rt
    err, pool = rt.cudaDeviceGetDefaultMemPool(device_index)
    assert err == rt.cudaError_t.cudaSuccess
    err, used = rt.cudaMemPoolGetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent)
    assert err == rt.cudaError_t.cudaSuccess
    return int(used)


def test_noalloc_allocates_no_device_memory(pkg, cuda):
    eng = pkg.get_engine(cuda)
    w = pkg.workloads.make_workload(1)
    coords = torch.from_numpy(w.coords).to(cuda)
    out = torch.empty((w.n, 27), dtype=torch.int32, device=cuda)
    lib = pkg._lib.lib()
    eng.bind_stream()
    call = lambda: lib.sc_kmap_build_noalloc(eng.handle, ctypes.c_void_p(coords.data_ptr()), w.n, 1,
                                             ctypes.c_void_p(out.data_ptr()))
    assert call() == pkg._lib.SC_OK  # warm call: the scratch address is looked up once
    torch.cuda.synchronize()
    free0, pool0, torch0 = torch.cuda.mem_get_info(cuda)[0], _pool_used(cuda.index), torch.cuda.memory_allocated(cuda)
    for _ in range(3):
        assert call() == pkg._lib.SC_OK
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(cuda)[0] == free0
    assert _pool_used(cuda.index) == pool0
    assert torch.cuda.memory_allocated(cuda) == torch0


def test_noalloc_empty_input_and_out_of_range_coords(pkg, cuda):
    eng = pkg.get_engine(cuda)
    st, _ = _noalloc(pkg, eng, torch.zeros((0, 4), dtype=torch.int32, device=cuda))
    assert st == pkg._lib.SC_OK
    bad = torch.tensor([[0, 1, 2, 3], [0, 70000, 0, 0]], dtype=torch.int32, device=cuda)
    st, _ = _noalloc(pkg, eng, bad)
    assert st == pkg._lib.SC_ERANGE
    w = pkg.workloads.make_workload(1, scale=0.5)  # usable afterwards
    c = torch.from_numpy(w.coords).to(cuda)
    st, got = _noalloc(pkg, eng, c)
    assert st == pkg._lib.SC_OK
    assert torch.equal(got, pkg.build_kmap(c, engine=eng).export())


def test_noalloc_refused_during_stream_capture(pkg, cuda):
    eng = pkg.get_engine(cuda)
    w = pkg.workloads.make_workload(1, scale=0.5)
    coords = torch.from_numpy(w.coords).to(cuda)
    out = torch.empty((w.n, 27), dtype=torch.int32, device=cuda)
    s = torch.cuda.Stream(cuda)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        g.capture_begin()
        try:
            out.zero_()  # the graph holds one node of its own
            eng.bind_stream()  # the handle now enqueues on the capturing stream
            st = pkg._lib.lib().sc_kmap_build_noalloc(eng.handle, ctypes.c_void_p(coords.data_ptr()), w.n, 1,
                                                      ctypes.c_void_p(out.data_ptr()))
        finally:
            g.capture_end()
    eng.bind_stream(torch.cuda.current_stream(cuda))
    assert st == pkg._lib.SC_EINVAL
    assert b"captured" in pkg._lib.lib().sc_last_error(eng.handle)
