"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and the Python binding covers the same set."""
import ctypes
import subprocess

import pytest


def test_library_loads_and_reports_version(pkg):
    v = pkg._lib.lib().sc_version()
    assert v.startswith(b"sparseconv_b200")


def test_every_header_symbol_is_exported(pkg):
    names = pkg._lib.header_symbols()
    assert len(names) >= 20
    L = pkg._lib.lib()
    for n in names:
        assert hasattr(L, n), f"{n} declared in the header but not exported"


def test_dynamic_symbol_table_matches_header(pkg):
    out = subprocess.run(["nm", "-D", "--defined-only", pkg._lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln and ln.split()[-1].startswith("sc_")}
    assert exported == set(pkg._lib.header_symbols())


def test_binding_covers_header(pkg):
    assert set(pkg._lib._SIGNATURES) == set(pkg._lib.header_symbols())


def test_null_arguments_are_rejected_without_touching_the_device(pkg):
    L = pkg._lib.lib()
    assert L.sc_create(None, None) == pkg._lib.SC_EINVAL
    assert L.sc_destroy(None) == pkg._lib.SC_EINVAL
    assert L.sc_kmap_build(None, None, 0, 3, 1, 0, None) == pkg._lib.SC_EINVAL
    assert L.sc_conv3d(None, None, None, None, None, None, None, 1, 1, 1, 0, 0.0) == pkg._lib.SC_EINVAL
    out = ctypes.c_void_p(1234)
    assert L.sc_kmap_concat(None, None, None, 0, ctypes.byref(out)) == pkg._lib.SC_EINVAL
    assert L.sc_conv3d_halo(None, None, None, None, None, None, None, 1, 1, 1, 0, 0.0, None, 2, 0, 1) == \
        pkg._lib.SC_EINVAL
    assert L.sc_halo_push(None, None, 16, None, None, None, 0, None, None, 2, 0, 1) == pkg._lib.SC_EINVAL
    assert L.sc_halo_wait(None, None, 2, 0, 1) == pkg._lib.SC_EINVAL
    assert L.sc_last_error(None) == b"null handle"
    cfg = pkg._lib.ScConfig()
    L.sc_config_default(ctypes.byref(cfg))
    assert (cfg.device, cfg.map_mode, cfg.debug_bounds) == (0, pkg._lib.SC_MAP_HASH, 0)


def test_create_without_gpu_fails_cleanly(pkg):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    st = pkg._lib.lib().sc_create(ctypes.byref(h), None)
    assert st in (pkg._lib.SC_ECUDA, pkg._lib.SC_EUNSUPPORTED)
    assert not h.value


def test_status_to_exception_mapping(pkg):
    L = pkg._lib
    with pytest.raises(L.DuplicateCoordError):
        L.check(L.SC_EDUP_COORD)
    with pytest.raises(L.CoordRangeError):
        L.check(L.SC_ERANGE)
    with pytest.raises(L.SparseConvError):
        L.check(L.SC_ETIMEOUT)
    L.check(L.SC_OK)
