"""CPU restatement of the reference sparse-conv path (TEST INFRASTRUCTURE ONLY).

This module is the checker for the CUDA engine.  Only the test suite, the
smoke check and the benchmark's CPU-baseline leg may import it; the engine
never routes through it.

Parity status: **parity unpinned** against the reference's own code.  The
reference repository ships the sparse conv only as WGSL compute shaders run
through Deno/WebGPU (``src/sparse/ops/conv3d_wgsl.ts``), which cannot run on
these machines, and its Python ``conv_none.py`` / ``hashmap_fallback.py``
live in an empty git submodule.  No golden vectors for this path exist in the
reference.  The restatement is therefore pinned to the two invariants the
reference documents for those modules (``README.md:80-81``):

* the neighbour map equals a brute-force dense-grid lookup (every self and
  neighbour lookup correct), and
* the sparse conv equals dense ``torch.nn.functional.conv3d`` sampled at the
  active voxels (to 1e-5 in fp32).

Both invariants are checked in ``tests/test_oracle.py``.

Functions and the reference lines they follow:

* ``kmap_bruteforce`` -- ``src/sparse/ops/conv3d_wgsl.ts:44-71`` (pass 0, dense
  ``sp_to_lin`` scatter) and ``:75-128`` (pass 1: offset order
  ``v = kd*Kh*Kw + kh*Kw + kw`` at ``:91-101``, kd on x / kh on y / kw on z at
  ``:115-117``, out-of-bounds -> -1 at ``:120``), with the batch column made
  part of the lookup (``src/sparse/sparse_tensor.ts:19``).
* ``kmap_sorted`` -- the ``flat_idx`` sort + ``searchsorted`` map described for
  ``hashmap_fallback.py`` (``README.md:111``).
* ``conv_gather`` -- pass 2's sum ``out[n,co] = b[co] + sum_v sum_ci
  f[map[n,v],ci] * W[co,v,ci]`` (``src/sparse/ops/conv3d_wgsl.ts:177-222``)
  with weight layout ``(Co,Kd,Kh,Kw,Ci)`` (``src/sparse/ops/conv3d.ts:5,48-49``),
  accumulated in float64.  The defects of that WGSL pass are not reproduced:
  its weight tile reads row ``tile + 2*local_co`` instead of
  ``tile + local_co`` (``conv3d_wgsl.ts:188-197,219``), it returns before a
  ``workgroupBarrier`` (``:174``), and it accumulates in f16 for f16 inputs
  (``:177``).
* ``down2_map`` / ``up2_map`` -- stride-2 2x2x2 down-sample and its transpose
  onto the fine coords; the reference's Python versions are absent, so the
  semantics are the ones fixed by the engine's contract (unique parents in
  ascending packed-key order; child slot ``(x&1)*4 + (y&1)*2 + (z&1)``).
* ``conv_depthwise`` / ``convnext_block`` -- the VAE decoder's ConvNeXt block
  (``src/models/sparse_unet_vae_decoder.ts:48-77``): conv -> LayerNorm ->
  Linear -> LayerNorm -> SiLU -> Linear + skip, with a depthwise
  ``(C,3,3,3,1)`` conv weight as an alternative to the dense one.
* ``subdivide2`` -- 2x2x2 voxel subdivision with an optional child mask, the
  upsample the TS decoder leaves out (``sparse_unet_vae_decoder.ts:155-175``).
* ``attention_varlen`` -- per-sequence scaled dot-product attention of the
  SLat flow model (``src/sparse/ops/attention.ts:24-80``).
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "flat_keys", "kmap_bruteforce", "kmap_sorted", "conv_gather", "down2_map",
    "up2_map", "layer_norm", "silu", "resblock", "round_bf16", "offsets27", "dense_conv3d_check",
    "torch_cpu_kmap", "torch_cpu_conv", "conv_depthwise", "convnext_block", "subdivide2", "attention_varlen",
]


def offsets27(dilation=1):
    """Offset table for a 3x3x3 kernel, ``v = kd*9 + kh*3 + kw``.

    Follows ``kernel_offset`` in ``src/sparse/ops/conv3d_wgsl.ts:91-101``:
    ``(kd - Kd/2) * dilD`` on x, ``(kh - Kh/2) * dilH`` on y, ``(kw - Kw/2) * dilW``
    on z.  ``dilation`` is one int or ``(dilD, dilH, dilW)``
    (``src/sparse/ops/conv3d.ts:43-45``).
    """
    dd, dh, dw = (dilation,) * 3 if np.isscalar(dilation) else tuple(int(d) for d in dilation)
    out = np.zeros((27, 3), np.int64)
    for v in range(27):
        kd, kh, kw = v // 9, (v // 3) % 3, v % 3
        out[v] = ((kd - 1) * dd, (kh - 1) * dh, (kw - 1) * dw)
    return out


def flat_keys(coords, spatial_shape):
    """``flat_idx = ((b*X + x)*Y + y)*Z + z`` as int64 (lexicographic order)."""
    c = np.asarray(coords).astype(np.int64)
    X, Y, Z = (int(s) for s in spatial_shape)
    return ((c[:, 0] * X + c[:, 1]) * Y + c[:, 2]) * Z + c[:, 3]


def kmap_bruteforce(coords, spatial_shape, batch_size, dilation=1):
    """Dense-grid neighbour map ``[N, 27]`` int32 (small grids only).

    Pass 0 writes ``grid[b, x, y, z] = i``; pass 1 reads the 27 neighbours with
    a bounds check.  Duplicate coords raise (the engine reports them as an
    error instead of the reference's last-writer-wins race).
    """
    c = np.asarray(coords).astype(np.int64)
    X, Y, Z = (int(s) for s in spatial_shape)
    grid = np.full((batch_size, X, Y, Z), -1, np.int32)
    n = len(c)
    if n:
        if np.any(grid[c[:, 0], c[:, 1], c[:, 2], c[:, 3]] != -1):
            raise ValueError("duplicate coordinate")
    # pass 0 (conv3d_wgsl.ts:60-69), batch-aware
    flat = ((c[:, 0] * X + c[:, 1]) * Y + c[:, 2]) * Z + c[:, 3]
    gflat = grid.reshape(-1)
    if len(np.unique(flat)) != n:
        raise ValueError("duplicate coordinate")
    gflat[flat] = np.arange(n, dtype=np.int32)
    # pass 1 (conv3d_wgsl.ts:106-127)
    out = np.full((n, 27), -1, np.int32)
    for v, (dx, dy, dz) in enumerate(offsets27(dilation)):
        nx, ny, nz = c[:, 1] + dx, c[:, 2] + dy, c[:, 3] + dz
        ok = (nx >= 0) & (nx < X) & (ny >= 0) & (ny < Y) & (nz >= 0) & (nz < Z)
        idx = np.where(ok)[0]
        out[idx, v] = gflat[((c[idx, 0] * X + nx[idx]) * Y + ny[idx]) * Z + nz[idx]]
    return out


def kmap_sorted(coords, spatial_shape, dilation=1, rows=None):
    """Sort + searchsorted neighbour map ``[N, 27]`` int32 (any size).

    ``rows`` (optional index array) restricts the output to those map rows,
    ``[len(rows), 27]``; neighbours are still looked up among all voxels.
    ``dilation`` is one int (all axes) or ``(dil_x, dil_y, dil_z)``."""
    c = np.asarray(coords).astype(np.int64)
    X, Y, Z = (int(s) for s in spatial_shape)
    keys = flat_keys(c, spatial_shape)
    order = np.argsort(keys, kind="stable")
    sk = keys[order]
    if len(sk) > 1 and np.any(sk[1:] == sk[:-1]):
        raise ValueError("duplicate coordinate")
    n = len(c)
    q_c = c if rows is None else c[np.asarray(rows)]
    out = np.full((len(q_c), 27), -1, np.int32)
    for v, (dx, dy, dz) in enumerate(offsets27(dilation)):
        nx, ny, nz = q_c[:, 1] + dx, q_c[:, 2] + dy, q_c[:, 3] + dz
        ok = (nx >= 0) & (nx < X) & (ny >= 0) & (ny < Y) & (nz >= 0) & (nz < Z)
        q = ((q_c[:, 0] * X + nx) * Y + ny) * Z + nz
        pos = np.searchsorted(sk, q)
        pos_c = np.minimum(pos, max(n - 1, 0))
        hit = ok & (pos < n) & (sk[pos_c] == q) if n else ok
        out[hit, v] = order[pos_c[hit]].astype(np.int32)
    return out


def conv_gather(feats, kmap, weight, bias=None, out_dtype=np.float64):
    """``out[n] = bias + sum_v W[:, v, :] @ feats[kmap[n, v]]`` over valid entries.

    ``weight`` is ``(Co, K..., Ci)`` (any number of kernel axes, flattened to K
    offsets); accumulation is float64.
    """
    f = np.asarray(feats, np.float64)
    W = np.asarray(weight, np.float64)
    co, ci = W.shape[0], W.shape[-1]
    W = W.reshape(co, -1, ci)
    K = W.shape[1]
    km = np.asarray(kmap)
    assert km.shape[1] == K, (km.shape, W.shape)
    out = np.zeros((km.shape[0], co), np.float64)
    if bias is not None:
        out += np.asarray(bias, np.float64)[None, :]
    for v in range(K):
        rows = np.where(km[:, v] >= 0)[0]
        if len(rows):
            out[rows] += f[km[rows, v]] @ W[:, v, :].T
    return out.astype(out_dtype)


def down2_map(coords):
    """Stride-2 2x2x2 down-sample map.

    Returns ``(parent_coords [Np,4] int32, dmap [Np,8] int32)``: parents are the
    unique ``(b, x>>1, y>>1, z>>1)`` in ascending lexicographic order and
    ``dmap[p, (x&1)*4 + (y&1)*2 + (z&1)]`` is the fine row of that child or -1.
    """
    c = np.asarray(coords).astype(np.int64)
    pc = np.stack([c[:, 0], c[:, 1] >> 1, c[:, 2] >> 1, c[:, 3] >> 1], 1)
    key = (((pc[:, 0] << 16 | pc[:, 1]) << 16 | pc[:, 2]) << 16) | pc[:, 3]
    uk, inv = np.unique(key, return_inverse=True)
    parents = np.stack([(uk >> 48) & 0xFFFF, (uk >> 32) & 0xFFFF, (uk >> 16) & 0xFFFF, uk & 0xFFFF], 1)
    slot = (c[:, 1] & 1) * 4 + (c[:, 2] & 1) * 2 + (c[:, 3] & 1)
    dmap = np.full((len(uk), 8), -1, np.int32)
    dmap[inv, slot] = np.arange(len(c), dtype=np.int32)
    return parents.astype(np.int32), dmap


def up2_map(coords, parent_coords=None):
    """Transposed 2x2x2 map onto the fine coords: ``umap[c, slot(c)] = parent(c)``."""
    c = np.asarray(coords).astype(np.int64)
    if parent_coords is None:
        parent_coords, _ = down2_map(coords)
    p = np.asarray(parent_coords).astype(np.int64)
    pkey = (((p[:, 0] << 16 | p[:, 1]) << 16 | p[:, 2]) << 16) | p[:, 3]
    ckey = (((c[:, 0] << 16 | (c[:, 1] >> 1)) << 16 | (c[:, 2] >> 1)) << 16) | (c[:, 3] >> 1)
    order = np.argsort(pkey)
    pos = np.searchsorted(pkey[order], ckey)
    pos = np.minimum(pos, len(p) - 1)
    found = pkey[order][pos] == ckey
    umap = np.full((len(c), 8), -1, np.int32)
    slot = (c[:, 1] & 1) * 4 + (c[:, 2] & 1) * 2 + (c[:, 3] & 1)
    rows = np.where(found)[0]
    umap[rows, slot[rows]] = order[pos[rows]].astype(np.int32)
    return umap


def layer_norm(x, eps=1e-6):
    """Row LayerNorm without affine (``src/dense/ops/layer_norm.ts:28-60``, eps as
    used by ``src/models/sparse_unet_vae_decoder.ts:62,68``)."""
    x = np.asarray(x, np.float64)
    mu = x.mean(1, keepdims=True)
    var = ((x - mu) ** 2).mean(1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps)


def silu(x):
    """``x * sigmoid(x)`` (``src/dense/ops/silu.ts:20-31``)."""
    x = np.asarray(x, np.float64)
    return x / (1.0 + np.exp(-x))


def round_bf16(x):
    """Rounds to the nearest bf16 value (ties to even), returned as float64.

    Used where the engine stores an intermediate in bf16 (the ResBlock's
    hidden activation, the activations between chained convs)."""
    a = np.ascontiguousarray(np.asarray(x, np.float64).astype(np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).astype(np.float64)


def resblock(feats, kmap, w1, b1, w2, b2, eps=1e-6, hidden_bf16=False):
    """conv -> LayerNorm -> SiLU -> conv, plus identity skip (float64).

    ``hidden_bf16`` rounds the hidden activation to bf16 between the convs,
    as an engine that stores it in bf16 does."""
    h = conv_gather(feats, kmap, w1, b1)
    h = silu(layer_norm(h, eps))
    if hidden_bf16:
        h = round_bf16(h)
    return conv_gather(h, kmap, w2, b2) + np.asarray(feats, np.float64)


def conv_depthwise(feats, kmap, weight, bias=None):
    """Depthwise conv ``out[n, c] = bias[c] + sum_v W[c, v] * feats[kmap[n, v], c]``.

    ``weight`` is ``(C, 3, 3, 3, 1)`` (or ``(C, 27)``), ``v = kd*9 + kh*3 + kw``
    as in ``src/sparse/ops/conv3d.ts:48-49``; float64."""
    f = np.asarray(feats, np.float64)
    W = np.asarray(weight, np.float64).reshape(f.shape[1], -1)
    km = np.asarray(kmap)
    out = np.zeros((km.shape[0], f.shape[1]), np.float64)
    if bias is not None:
        out += np.asarray(bias, np.float64)[None, :]
    for v in range(km.shape[1]):
        rows = np.where(km[:, v] >= 0)[0]
        if len(rows):
            out[rows] += f[km[rows, v]] * W[None, :, v]
    return out


def convnext_block(feats, kmap, dw_weight, dw_bias, l0_weight, l0_bias, l2_weight, l2_bias, eps=1e-6,
                   round_to_bf16=False):
    """Sparse ConvNeXt block of the VAE decoder
    (``src/models/sparse_unet_vae_decoder.ts:48-77``): dw_conv -> LayerNorm ->
    Linear0 -> LayerNorm -> SiLU -> Linear2, plus identity skip (float64).

    ``dw_weight`` ``(C, 3, 3, 3, C)`` is a full conv, ``(C, 3, 3, 3, 1)`` a
    depthwise one, None skips the conv.  Linear weights are ``(out, in)``
    (``torch.nn.Linear``), i.e. ``x @ W.T``.  ``round_to_bf16`` rounds every
    intermediate the engine stores in bf16 (conv output after LayerNorm, the
    Linear0 output, the activation after SiLU)."""
    f = np.asarray(feats, np.float64)
    rnd = round_bf16 if round_to_bf16 else (lambda a: a)
    if dw_weight is None:
        h = f
    elif np.asarray(dw_weight).shape[-1] == 1 and f.shape[1] != 1:
        h = rnd(conv_depthwise(f, kmap, dw_weight, dw_bias))
    else:
        h = conv_gather(f, kmap, dw_weight, dw_bias)
    h = rnd(layer_norm(h, eps))
    h = h @ np.asarray(l0_weight, np.float64).T
    if l0_bias is not None:
        h = h + np.asarray(l0_bias, np.float64)[None, :]
    h = rnd(silu(layer_norm(rnd(h), eps)))
    h = h @ np.asarray(l2_weight, np.float64).T
    if l2_bias is not None:
        h = h + np.asarray(l2_bias, np.float64)[None, :]
    return h + f


def subdivide2(coords, feats, child_mask=None):
    """2x2x2 subdivision: each voxel ``(b, x, y, z)`` becomes its children
    ``(b, 2x+i, 2y+j, 2z+k)``, child ``s = i*4 + j*2 + k``, rows in
    (parent, s) order, each carrying its parent's features.  ``child_mask``
    (``[N, 8]`` bool) keeps only the marked children.

    The TS decoder only doubles ``spatialShape`` and keeps the coords
    (``src/models/sparse_unet_vae_decoder.ts:155-175``); the subdividing
    module it stands in for (TRELLIS ``SparseSubdivide`` / the
    ``SparseResBlockUpsample3d`` subdivision mask) lives in the ``trellis2``
    submodule, absent from the tree, and is restated here from its published
    behaviour."""
    c = np.asarray(coords, np.int64)
    n = c.shape[0]
    s = np.arange(8)
    off = np.stack([(s >> 2) & 1, (s >> 1) & 1, s & 1], 1)
    fine = np.empty((n, 8, 4), np.int64)
    fine[:, :, 0] = c[:, None, 0]
    fine[:, :, 1:] = 2 * c[:, None, 1:] + off[None]
    parent = np.repeat(np.arange(n), 8).reshape(n, 8)
    keep = np.ones((n, 8), bool) if child_mask is None else np.asarray(child_mask, bool).reshape(n, 8)
    fine, parent = fine[keep], parent[keep]
    return fine.astype(np.int32), None if feats is None else np.asarray(feats)[parent]


def attention_varlen(q, k, v, cu_seqlens_q, cu_seqlens_kv=None, scale=None):
    """Per-sequence scaled dot-product attention, float64
    (``src/sparse/ops/attention.ts:24-80``: each batch item runs
    ``O = softmax(Q K^T * scale) V`` of ``src/dense/ops/attention.ts:2,61``
    with ``scale = 1 / sqrt(D)``; items with no query or no key rows are
    skipped and keep zeros, ``:50``).  ``q`` ``(N, H, D)``, ``k``/``v``
    ``(N_kv, H, D)``."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    cq = [int(x) for x in cu_seqlens_q]
    ck = cq if cu_seqlens_kv is None else [int(x) for x in cu_seqlens_kv]
    d = q.shape[2]
    s = 1.0 / np.sqrt(d) if scale is None else float(scale)
    out = np.zeros_like(q)
    for b in range(len(cq) - 1):
        qs, ks = q[cq[b]:cq[b + 1]], k[ck[b]:ck[b + 1]]
        if len(qs) == 0 or len(ks) == 0:
            continue
        logits = np.einsum("ihd,jhd->hij", qs, ks) * s
        logits -= logits.max(axis=2, keepdims=True)
        p = np.exp(logits)
        p /= p.sum(axis=2, keepdims=True)
        out[cq[b]:cq[b + 1]] = np.einsum("hij,jhd->ihd", p, v[ck[b]:ck[b + 1]])
    return out


def dense_conv3d_check(coords, feats, weight, bias, spatial_shape, batch_size):
    """Dense ``F.conv3d`` (padding 1) sampled at the active voxels (float64).

    Weight ``(Co,Kd,Kh,Kw,Ci)`` is permuted to torch's ``(Co,Ci,Kd,Kh,Kw)``;
    x pairs with Kd, y with Kh, z with Kw.
    """
    import torch
    import torch.nn.functional as F
    c = torch.as_tensor(np.asarray(coords).astype(np.int64))
    X, Y, Z = (int(s) for s in spatial_shape)
    ci = feats.shape[1]
    dense = torch.zeros((batch_size, ci, X, Y, Z), dtype=torch.float64)
    dense[c[:, 0], :, c[:, 1], c[:, 2], c[:, 3]] = torch.as_tensor(np.asarray(feats, np.float64))
    w = torch.as_tensor(np.asarray(weight, np.float64)).permute(0, 4, 1, 2, 3).contiguous()
    b = None if bias is None else torch.as_tensor(np.asarray(bias, np.float64))
    y = F.conv3d(dense, w, b, padding=1)
    return y[c[:, 0], :, c[:, 1], c[:, 2], c[:, 3]].numpy()


# ---------------------------------------------------------------------------
# torch-CPU versions used for the timed CPU baseline (same math, multithreaded)
# ---------------------------------------------------------------------------

def torch_cpu_kmap(coords_t, spatial_shape, dilation=1):
    """flat_idx sort + searchsorted on torch CPU tensors -> ``[N,27]`` int32."""
    import torch
    c = coords_t.to(torch.int64)
    X, Y, Z = (int(s) for s in spatial_shape)
    keys = ((c[:, 0] * X + c[:, 1]) * Y + c[:, 2]) * Z + c[:, 3]
    sk, order = torch.sort(keys)
    n = c.shape[0]
    out = torch.full((n, 27), -1, dtype=torch.int32)
    for v, (dx, dy, dz) in enumerate(offsets27(dilation).tolist()):
        nx, ny, nz = c[:, 1] + dx, c[:, 2] + dy, c[:, 3] + dz
        ok = (nx >= 0) & (nx < X) & (ny >= 0) & (ny < Y) & (nz >= 0) & (nz < Z)
        q = ((c[:, 0] * X + nx) * Y + ny) * Z + nz
        pos = torch.searchsorted(sk, q).clamp_(max=n - 1)
        hit = ok & (sk[pos] == q)
        out[:, v] = torch.where(hit, order[pos].to(torch.int32), torch.full_like(out[:, v], -1))
    return out


def torch_cpu_conv(feats_t, kmap_t, weight_t, bias_t=None):
    """27 x (index_select -> matmul -> index_add_) in float32 on torch CPU."""
    import torch
    co, ci = weight_t.shape[0], weight_t.shape[-1]
    W = weight_t.reshape(co, -1, ci)
    out = torch.zeros((kmap_t.shape[0], co), dtype=torch.float32)
    if bias_t is not None:
        out += bias_t.float()[None, :]
    f = feats_t.float()
    for v in range(W.shape[1]):
        col = kmap_t[:, v]
        rows = torch.nonzero(col >= 0).squeeze(1)
        if rows.numel():
            g = f.index_select(0, col[rows].long())
            out.index_add_(0, rows, g @ W[:, v, :].float().T)
    return out
