"""The reference's on-disk voxel cache: raw ``.coords.bin`` / ``.attrs.bin`` dumps.

The pipeline caches the sparse structure it meshes as two headerless ndarray
dumps (``trellis_webgpu.ts:8-9,42-43,80-88``; ``src/pipeline/run.ts:233-255``):

* ``{output}.coords.bin``: int32, row-major, ``(N, 3)`` ``[x, y, z]`` as the
  mesh pipeline reads it (``src/mesh/pipeline.ts:18,266``).  The Python side
  dumps whatever ``data["coords"]`` holds, so a ``(N, 4)`` ``[b, x, y, z]``
  dump is accepted too when the row count says so.
* ``{output}.attrs.bin``: float32, row-major, ``(N, C)``; the layout the
  pipeline uses is :data:`ATTR_LAYOUT` (``trellis_webgpu.ts:124``).

Files are little-endian (``ndarray.tofile`` on x86).  :func:`load_sparse`
turns a cache into this engine's ``(N, 4)`` int32 device coords (batch 0 for
3-column dumps) plus features, ready for :func:`build_kmap`.
"""
from __future__ import annotations

import os

import numpy as np

__all__ = ["ATTR_LAYOUT", "read_coords_bin", "read_attrs_bin", "write_coords_bin", "write_attrs_bin", "read_cache",
           "write_cache", "load_sparse"]

ATTR_LAYOUT = {"base_color": (0, 3), "metallic": 3, "roughness": 4, "alpha": 5}
DEFAULT_ATTR_CHANNELS = 6


def _read(path, dtype):
    data = np.fromfile(path, dtype=np.dtype(dtype).newbyteorder("<"))
    return data.astype(dtype, copy=False)


def read_coords_bin(path, columns=3):
    """``(N, columns)`` int32 coords from a raw dump; ``columns`` 3 or 4."""
    if columns not in (3, 4):
        raise ValueError("columns must be 3 ([x, y, z]) or 4 ([b, x, y, z])")
    flat = _read(path, np.int32)
    if flat.size % columns:
        raise ValueError(f"{path}: {flat.size} int32 values is not a whole number of {columns}-column rows")
    return flat.reshape(-1, columns)


def read_attrs_bin(path, channels=DEFAULT_ATTR_CHANNELS):
    """``(N, channels)`` float32 attributes from a raw dump."""
    flat = _read(path, np.float32)
    if channels <= 0 or flat.size % channels:
        raise ValueError(f"{path}: {flat.size} float32 values is not a whole number of {channels}-channel rows")
    return flat.reshape(-1, channels)


def _write(path, arr, dtype):
    a = np.ascontiguousarray(np.asarray(arr), dtype=np.dtype(dtype).newbyteorder("<"))
    tmp = f"{path}.tmp{os.getpid()}"
    a.tofile(tmp)
    os.replace(tmp, path)


def write_coords_bin(path, coords):
    """Raw int32 dump of ``(N, 3)`` or ``(N, 4)`` coords (written whole, then renamed)."""
    c = np.asarray(coords)
    if c.ndim != 2 or c.shape[1] not in (3, 4):
        raise ValueError("coords must be (N, 3) or (N, 4)")
    _write(path, c, np.int32)


def write_attrs_bin(path, attrs):
    """Raw float32 dump of ``(N, C)`` attributes."""
    a = np.asarray(attrs)
    if a.ndim != 2:
        raise ValueError("attrs must be (N, C)")
    _write(path, a, np.float32)


def read_cache(prefix, channels=DEFAULT_ATTR_CHANNELS, columns=None):
    """``(coords, attrs)`` from ``{prefix}.coords.bin`` / ``{prefix}.attrs.bin``.

    ``columns`` None infers 3 or 4 from the attribute row count; a dump that
    fits neither raises ``ValueError``."""
    attrs = read_attrs_bin(f"{prefix}.attrs.bin", channels)
    n = attrs.shape[0]
    if columns is None:
        size = os.path.getsize(f"{prefix}.coords.bin") // 4
        if size == 3 * n:
            columns = 3
        elif size == 4 * n:
            columns = 4
        else:
            raise ValueError(f"{prefix}.coords.bin holds {size} int32 values, neither 3 nor 4 per attribute row ({n})")
    coords = read_coords_bin(f"{prefix}.coords.bin", columns)
    if coords.shape[0] != n:
        raise ValueError(f"{coords.shape[0]} coords rows but {n} attribute rows")
    return coords, attrs


def write_cache(prefix, coords, attrs):
    """Writes ``{prefix}.coords.bin`` and ``{prefix}.attrs.bin``."""
    if np.asarray(coords).shape[0] != np.asarray(attrs).shape[0]:
        raise ValueError("coords and attrs must have the same number of rows")
    write_coords_bin(f"{prefix}.coords.bin", coords)
    write_attrs_bin(f"{prefix}.attrs.bin", attrs)


def load_sparse(prefix, device="cuda", channels=DEFAULT_ATTR_CHANNELS, batch=0, feat_dtype=None, pad_channels=1):
    """A cache as a :class:`SparseTensor` on ``device``: ``(N, 4)`` int32
    ``[b, x, y, z]`` coords (``batch`` for 3-column dumps) and the attributes
    as features (``feat_dtype``, default float32), zero-padded to a multiple of
    ``pad_channels`` columns (8 for the depthwise conv, 16 for the bf16
    tensor-core conv)."""
    import torch

    from .sparse_conv import SparseTensor

    coords, attrs = read_cache(prefix, channels)
    if coords.shape[1] == 3:
        coords = np.concatenate([np.full((coords.shape[0], 1), batch, np.int32), coords], 1)
    if coords.size and (coords.min() < 0):
        raise ValueError("negative coordinates in the cache")
    c = attrs.shape[1]
    cp = -(-c // pad_channels) * pad_channels
    if cp != c:
        attrs = np.concatenate([attrs, np.zeros((attrs.shape[0], cp - c), np.float32)], 1)
    t_c = torch.from_numpy(np.ascontiguousarray(coords)).to(device)
    t_f = torch.from_numpy(np.ascontiguousarray(attrs)).to(device, feat_dtype or torch.float32)
    return SparseTensor(t_f, t_c)
