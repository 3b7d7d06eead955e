"""The raw `.coords.bin` / `.attrs.bin` voxel cache (no GPU)."""
import numpy as np
import pytest


def test_round_trip_three_columns(pkg, tmp_path):
    rng = np.random.default_rng(1)
    coords = rng.integers(0, 512, (1000, 3)).astype(np.int32)
    attrs = rng.random((1000, 6)).astype(np.float32)
    prefix = str(tmp_path / "out.glb")
    pkg.coords_io.write_cache(prefix, coords, attrs)
    # the files are headerless little-endian dumps, as ndarray.tofile writes them
    assert (tmp_path / "out.glb.coords.bin").stat().st_size == 1000 * 3 * 4
    assert np.array_equal(np.fromfile(prefix + ".coords.bin", "<i4").reshape(-1, 3), coords)
    c, a = pkg.coords_io.read_cache(prefix)
    assert c.dtype == np.int32 and c.shape == (1000, 3) and np.array_equal(c, coords)
    assert a.dtype == np.float32 and np.array_equal(a, attrs)


def test_four_column_dump_is_inferred(pkg, tmp_path):
    rng = np.random.default_rng(2)
    coords = np.concatenate([np.zeros((50, 1), np.int32), rng.integers(0, 64, (50, 3)).astype(np.int32)], 1)
    prefix = str(tmp_path / "x")
    pkg.coords_io.write_cache(prefix, coords, rng.random((50, 6)))
    c, _ = pkg.coords_io.read_cache(prefix)
    assert c.shape == (50, 4) and np.array_equal(c, coords)


def test_bad_sizes_raise(pkg, tmp_path):
    prefix = str(tmp_path / "bad")
    np.arange(10, dtype=np.int32).tofile(prefix + ".coords.bin")
    np.zeros(12, np.float32).tofile(prefix + ".attrs.bin")      # 2 rows of 6
    with pytest.raises(ValueError, match="neither 3 nor 4"):
        pkg.coords_io.read_cache(prefix)
    with pytest.raises(ValueError, match="whole number"):
        pkg.coords_io.read_coords_bin(prefix + ".coords.bin", 3)
    with pytest.raises(ValueError, match="whole number"):
        pkg.coords_io.read_attrs_bin(prefix + ".attrs.bin", 5)
    with pytest.raises(ValueError):
        pkg.coords_io.write_cache(prefix, np.zeros((3, 3), np.int32), np.zeros((2, 6)))
    with pytest.raises(ValueError):
        pkg.coords_io.write_coords_bin(prefix + ".c", np.zeros((3, 2), np.int32))


def test_empty_cache(pkg, tmp_path):
    prefix = str(tmp_path / "empty")
    pkg.coords_io.write_cache(prefix, np.zeros((0, 3), np.int32), np.zeros((0, 6), np.float32))
    c, a = pkg.coords_io.read_cache(prefix)
    assert c.shape == (0, 3) and a.shape == (0, 6)


def test_attr_layout_matches_pipeline(pkg):
    assert pkg.coords_io.ATTR_LAYOUT == {"base_color": (0, 3), "metallic": 3, "roughness": 4, "alpha": 5}
