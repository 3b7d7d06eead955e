"""Seeded synthetic sparse-voxel workloads C1..C5.

The five configurations are the ones the engine is measured and checked on:
ellipsoid shells (and unions of shells) voxelised on a cubic grid, with
features and weights drawn from seeded normal distributions.  The reference
pipeline produces its sparse structures from a flow model that is not part of
this path, so these seeded shapes stand in for them: surface-like active sets
(1-2 voxels thick), batch-sorted coords, Morton order inside each batch.

Coordinates follow the reference SparseTensor convention
(``src/sparse/sparse_tensor.ts:19``): int32 rows ``[b, x, y, z]``.
Weights follow the checkpoint layout ``(Co, Kd, Kh, Kw, Ci)``
(``src/sparse/ops/conv3d.ts:5,19``).

Every generator is pure numpy with an explicit ``numpy.random.Generator``,
so the same seed gives the same voxels on every machine.
"""
from __future__ import annotations

import dataclasses
import numpy as np

__all__ = [
    "Workload", "CONFIGS", "make_workload", "ellipsoid_shell", "morton_codes",
    "morton_sort", "shuffle_rows", "count_pairs",
]


def _shell_columns(cx, cy, cz, a, b, c, h, grid, xa=None, xb=None):
    """Candidate (x, y, z) voxels near the surface of one axis-aligned ellipsoid.

    Candidates are every voxel of each (x, y) column that lies inside the
    ellipsoid grown by ``h + 2`` and outside the ellipsoid shrunk by ``h + 2``
    (two z windows per column), so the interior is never enumerated.  ``xa``,
    ``xb`` restrict the columns to the x range [xa, xb].
    """
    m = h + 2.0
    x0 = max(0, int(np.floor(cx - a - m))) if xa is None else xa
    x1 = min(grid - 1, int(np.ceil(cx + a + m))) if xb is None else xb
    y0 = max(0, int(np.floor(cy - b - m)))
    y1 = min(grid - 1, int(np.ceil(cy + b + m)))
    xs = np.arange(x0, x1 + 1, dtype=np.float64)
    ys = np.arange(y0, y1 + 1, dtype=np.float64)
    X, Y = np.meshgrid(xs, ys, indexing="ij")
    X = X.ravel()
    Y = Y.ravel()
    ao, bo, co = a + m, b + m, c + m
    to = ((X - cx) / ao) ** 2 + ((Y - cy) / bo) ** 2
    keep = to <= 1.0
    X, Y = X[keep], Y[keep]
    ho = co * np.sqrt(np.maximum(0.0, 1.0 - to[keep]))
    ai, bi, ci = max(a - m, 0.0), max(b - m, 0.0), max(c - m, 0.0)
    if ai > 0 and bi > 0 and ci > 0:
        ti = ((X - cx) / ai) ** 2 + ((Y - cy) / bi) ** 2
        hi = np.where(ti < 1.0, ci * np.sqrt(np.maximum(0.0, 1.0 - ti)), -1.0)
    else:
        hi = np.full_like(X, -1.0)
    zlo = np.maximum(0, np.floor(cz - ho)).astype(np.int64)
    zhi = np.minimum(grid - 1, np.ceil(cz + ho)).astype(np.int64)
    # inner exclusion window [ilo, ihi] (empty when hi < 0)
    ilo = np.where(hi >= 0, np.ceil(cz - hi), zhi + 1).astype(np.int64)
    ihi = np.where(hi >= 0, np.floor(cz + hi), zhi).astype(np.int64)
    # window 1: [zlo, min(ilo-1, zhi)], window 2: [max(ihi+1, zlo), zhi] when inner exists
    w1_hi = np.minimum(ilo - 1, zhi)
    w2_lo = np.where(hi >= 0, np.maximum(ihi + 1, zlo), zhi + 1)
    out = []
    for lo, hi_ in ((zlo, w1_hi), (w2_lo, zhi)):
        n = np.maximum(0, hi_ - lo + 1)
        tot = int(n.sum())
        if tot == 0:
            continue
        rep_x = np.repeat(X, n)
        rep_y = np.repeat(Y, n)
        starts = np.repeat(lo, n)
        offs = np.arange(tot) - np.repeat(np.cumsum(n) - n, n)
        out.append(np.stack([rep_x, rep_y, (starts + offs).astype(np.float64)], 1))
    if not out:
        return np.zeros((0, 3), np.float64)
    return np.concatenate(out, 0)


def ellipsoid_shell(centre, axes, half_thickness, grid):
    """Integer voxels whose first-order distance to the ellipsoid surface is <= h.

    The distance is ``F(p) / |grad F(p)|`` with ``F(p) = sum(((p-c)/a)^2) - 1``,
    evaluated at voxel coordinates.  Returns an ``(n, 3)`` int32 array.
    """
    cx, cy, cz = (float(v) for v in centre)
    a, b, c = (float(v) for v in axes)
    # x slabs of 32 columns keep the float64 temporaries small; the voxel set
    # does not depend on the slab size
    m = half_thickness + 2.0
    x0 = max(0, int(np.floor(cx - a - m)))
    x1 = min(grid - 1, int(np.ceil(cx + a + m)))
    parts = []
    for xs in range(x0, x1 + 1, 32):
        P = _shell_columns(cx, cy, cz, a, b, c, half_thickness, grid, xs, min(xs + 31, x1))
        if len(P) == 0:
            continue
        d = P - np.array([cx, cy, cz])
        ax = np.array([a, b, c])
        F = np.sum((d / ax) ** 2, 1) - 1.0
        g = 2.0 * d / ax ** 2
        gn = np.sqrt(np.sum(g * g, 1))
        dist = np.abs(F) / np.maximum(gn, 1e-12)
        parts.append(P[dist <= half_thickness].astype(np.int32))
    if not parts:
        return np.zeros((0, 3), np.int32)
    return np.concatenate(parts, 0)


def _part1by2(v):
    v = v.astype(np.uint64) & np.uint64(0x1FFFFF)
    v = (v | (v << np.uint64(32))) & np.uint64(0x1F00000000FFFF)
    v = (v | (v << np.uint64(16))) & np.uint64(0x1F0000FF0000FF)
    v = (v | (v << np.uint64(8))) & np.uint64(0x100F00F00F00F00F)
    v = (v | (v << np.uint64(4))) & np.uint64(0x10C30C30C30C30C3)
    v = (v | (v << np.uint64(2))) & np.uint64(0x1249249249249249)
    return v


def morton_codes(coords):
    """64-bit Morton code of ``(x, y, z)`` (21 bits each), x in the highest lane."""
    c = np.asarray(coords)
    return (_part1by2(c[:, 1]) << np.uint64(2)) | (_part1by2(c[:, 2]) << np.uint64(1)) | _part1by2(c[:, 3])


def morton_sort(coords):
    """Order rows by (batch, Morton(x, y, z)); returns the permutation."""
    c = np.asarray(coords)
    return np.lexsort((morton_codes(c), c[:, 0].astype(np.int64)))


def shuffle_rows(n, seed):
    """Seeded permutation used to present rows in random order to map tests."""
    return np.random.default_rng(1000 + seed).permutation(n)


@dataclasses.dataclass
class Workload:
    name: str
    coords: np.ndarray           # (N, 4) int32 [b, x, y, z]
    spatial_shape: tuple         # (X, Y, Z)
    batch_size: int
    feats: np.ndarray            # (N, Ci) float32 (cast to the compute dtype by the caller)
    weight: np.ndarray           # (Co, 3, 3, 3, Ci) float32  (or (Co,2,2,2,Ci))
    bias: np.ndarray             # (Co,) float32
    ci: int
    co: int
    dtype: str                   # "f32" | "bf16"
    extra: dict = dataclasses.field(default_factory=dict)

    @property
    def n(self):
        return int(self.coords.shape[0])


def _union(parts, batch):
    allp = np.concatenate(parts, 0) if parts else np.zeros((0, 3), np.int32)
    key = (allp[:, 0].astype(np.int64) << 40) | (allp[:, 1].astype(np.int64) << 20) | allp[:, 2].astype(np.int64)
    _, idx = np.unique(key, return_index=True)
    u = allp[np.sort(idx)]
    b = np.full((len(u), 1), batch, np.int32)
    return np.concatenate([b, u.astype(np.int32)], 1)


def _finish(coords):
    order = morton_sort(coords)
    return np.ascontiguousarray(coords[order].astype(np.int32))


def _normal(rng, shape, var):
    return (rng.standard_normal(shape) * np.sqrt(var)).astype(np.float32)


def _c1(rng, scale):
    grid = 64
    axes = rng.uniform(18 * scale, 30 * scale, 3)
    vox = ellipsoid_shell((32, 32, 32), axes, 1.0, grid)
    coords = _finish(_union([vox], 0))
    ci = co = 64
    return Workload("c1_64cube_f32_64to64", coords, (grid,) * 3, 1,
                    rng.standard_normal((len(coords), ci)).astype(np.float32),
                    _normal(rng, (co, 3, 3, 3, ci), 1.0 / (27 * ci)),
                    _normal(rng, (co,), 0.01), ci, co, "f32", {"axes": axes.tolist()})


def _shell_union(rng, grid, nshell, amin, amax, cmin, cmax, h):
    parts, meta = [], []
    for _ in range(nshell):
        axes = rng.uniform(amin, amax, 3)
        centre = rng.uniform(cmin, cmax, 3)
        parts.append(ellipsoid_shell(centre, axes, h, grid))
        meta.append((centre.tolist(), axes.tolist()))
    return parts, meta


def _c2(rng, scale):
    grid = 256
    parts, meta = _shell_union(rng, grid, 6, 55 * scale, 100 * scale, 100, 156, 0.5)
    coords = _finish(_union(parts, 0))
    ci = co = 128
    return Workload("c2_256cube_bf16_128to128", coords, (grid,) * 3, 1,
                    rng.standard_normal((len(coords), ci)).astype(np.float32),
                    _normal(rng, (co, 3, 3, 3, ci), 1.0 / (27 * ci)),
                    np.zeros((co,), np.float32), ci, co, "bf16", {"shells": meta})


def _c3(rng, scale):
    grid = 128
    rows = []
    meta = []
    for bidx in range(4):
        axes = rng.uniform(45 * scale, 62 * scale, 3)
        vox = ellipsoid_shell((64, 64, 64), axes, 0.5, grid)
        c = _union([vox], bidx)
        rows.append(c[morton_sort(c)])
        meta.append(axes.tolist())
    coords = np.ascontiguousarray(np.concatenate(rows, 0).astype(np.int32))
    ch = 256
    return Workload("c3_resblock_4x128cube_bf16_256", coords, (grid,) * 3, 4,
                    rng.standard_normal((len(coords), ch)).astype(np.float32),
                    _normal(rng, (ch, 3, 3, 3, ch), 1.0 / (27 * ch)),
                    np.zeros((ch,), np.float32), ch, ch, "bf16",
                    {"axes": meta,
                     "weight2": _normal(rng, (ch, 3, 3, 3, ch), 1.0 / (27 * ch)),
                     "bias2": np.zeros((ch,), np.float32)})


def _c4(rng, scale):
    grid = 512
    parts, meta = _shell_union(rng, grid, 6, 110 * scale, 200 * scale, 200, 312, 0.5)
    coords = _finish(_union(parts, 0))
    return Workload("c4_512cube_bf16_downsubup", coords, (grid,) * 3, 1,
                    rng.standard_normal((len(coords), 64)).astype(np.float32),
                    _normal(rng, (128, 2, 2, 2, 64), 1.0 / (8 * 64)),
                    np.zeros((128,), np.float32), 64, 128, "bf16",
                    {"shells": meta,
                     "w_sub": _normal(rng, (128, 3, 3, 3, 128), 1.0 / (27 * 128)),
                     "w_up": _normal(rng, (64, 2, 2, 2, 128), 1.0 / (8 * 128))})


def _c5(rng, scale):
    grid = 1024
    parts, meta = _shell_union(rng, grid, 4, 250 * scale, 420 * scale, 440, 584, 0.5)
    shell = _union(parts, 0)
    # 5% uniform interior fill: random voxels inside the first ellipsoid
    nfill = int(0.05 * len(shell))
    fills = []
    got = 0
    while got < nfill:
        centre, axes = meta[rng.integers(len(meta))]
        p = rng.uniform(-1, 1, (nfill * 2, 3))
        p = p[np.sum(p * p, 1) < 1.0]
        v = np.rint(np.asarray(centre) + p * np.asarray(axes)).astype(np.int64)
        v = v[np.all((v >= 0) & (v < grid), 1)]
        fills.append(v.astype(np.int32))
        got += len(v)
    fill = np.concatenate(fills, 0)[:nfill]
    coords = _finish(_union([shell[:, 1:], fill], 0))
    ch = 32
    # float32 normals drawn directly: 6M x 32 float64 draws took most of the
    # generation time (and 1.5 GB of temporaries)
    return Workload("c5_1024cube_bf16_32to32", coords, (grid,) * 3, 1,
                    rng.standard_normal((len(coords), ch), dtype=np.float32),
                    _normal(rng, (ch, 3, 3, 3, ch), 1.0 / (27 * ch)),
                    np.zeros((ch,), np.float32), ch, ch, "bf16", {"shells": meta})


CONFIGS = {1: _c1, 2: _c2, 3: _c3, 4: _c4, 5: _c5}


def make_workload(index, scale=1.0, seed=None):
    """Build configuration ``index`` (1..5).

    ``scale`` shrinks the ellipsoid axes (used by tests to make small cases
    with the same structure); ``seed`` defaults to the configuration index.
    """
    rng = np.random.default_rng(index if seed is None else seed)
    return CONFIGS[index](rng, scale)


def count_pairs(kmap):
    """M = number of valid (output, offset) pairs in an ``[N, K]`` map."""
    return int(np.count_nonzero(np.asarray(kmap) >= 0))
