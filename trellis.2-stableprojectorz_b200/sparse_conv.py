"""Host-side mirror of the reference sparse-conv operator, backed by the C ABI.

The names follow the reference:

* ``SparseTensor`` -- coords ``(N, 4)`` int32 ``[b, x, y, z]``, feats ``(N, C)``,
  a scale-keyed spatial cache shared by ``replace()``
  (``src/sparse/sparse_tensor.ts:18-121``).
* ``SparseConv3d(weight, bias, kernel_size, dilation).forward(x)`` -- weight in
  the checkpoint layout ``(Co, Kd, Kh, Kw, Ci)``; the neighbour map is cached in
  ``x``'s spatial cache under ``conv_neighbors_{Kw}x{Kh}x{Kd}_dil{..}`` exactly
  like ``src/sparse/ops/conv3d.ts:63-72,144-148``; returns ``x.replace(out)``.
* ``sparse_conv3d_forward(feats, coords, weight, bias)`` -- the function-level
  entry a ``SPARSE_CONV_BACKEND`` module exposes (the role of ``conv_none.py``).

Everything runs on the CUDA library; there is no CPU path.  Errors from the
library surface as ``SparseConvError`` (``DuplicateCoordError`` /
``CoordRangeError`` for bad coordinates).
"""
from __future__ import annotations

import collections
import math
import ctypes
import threading

import torch

from . import _lib as L
from ._lib import SparseConvError, DuplicateCoordError, CoordRangeError  # noqa: F401

__all__ = [
    "Engine", "get_engine", "KernelMap", "build_kmap", "build_down2", "build_up2", "conv3d",
    "SparseTensor", "SparseConv3d", "SparseConvDown2", "SparseConvUp2", "sparse_conv3d_forward",
    "sparse_resblock", "layernorm_silu",
]

_DTYPES = {torch.float32: L.SC_F32, torch.bfloat16: L.SC_BF16, torch.float16: L.SC_F16}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(None)


class Engine:
    """One library handle per CUDA device (``sc_create``); binds torch's current stream per call."""

    def __init__(self, device=None, map_mode="hash", debug_bounds=False):
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if dev.type != "cuda":
            raise ValueError("the sparse-conv engine runs on CUDA devices only")
        self.device = torch.device("cuda", dev.index if dev.index is not None else torch.cuda.current_device())
        self.lib = L.lib()
        cfg = L.ScConfig()
        self.lib.sc_config_default(ctypes.byref(cfg))
        cfg.device = self.device.index
        cfg.map_mode = {"hash": L.SC_MAP_HASH, "sort": L.SC_MAP_SORT}[map_mode]
        cfg.debug_bounds = 1 if debug_bounds else 0
        h = ctypes.c_void_p()
        st = self.lib.sc_create(ctypes.byref(h), ctypes.byref(cfg))
        if st != L.SC_OK:
            raise SparseConvError(st, f"sc_create failed on {self.device}")
        self.handle = h
        self.map_mode = map_mode

    def bind_stream(self, stream=None):
        s = torch.cuda.current_stream(self.device) if stream is None else stream
        self.lib.sc_set_stream(self.handle, ctypes.c_void_p(s.cuda_stream))

    def check(self, status, what=""):
        L.check(status, self.handle, what)

    def set_conv_ctas(self, max_ctas=0):
        """CTAs of the persistent conv (0 = one per SM); fewer leave SMs for a concurrent collective."""
        self.check(self.lib.sc_set_conv_ctas(self.handle, int(max_ctas)), "sc_set_conv_ctas")

    def launch_count(self):
        """Kernels launched through this handle so far."""
        return int(self.lib.sc_launch_count(self.handle))

    def synchronize(self):
        self.check(self.lib.sc_synchronize(self.handle), "synchronize")

    def close(self):
        if getattr(self, "handle", None):
            self.lib.sc_destroy(self.handle)
            self.handle = None


_engines = {}
_engines_lock = threading.Lock()


def get_engine(device=None, map_mode="hash"):
    """Cached Engine for ``(device, map_mode)``."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    key = (idx, map_mode)
    with _engines_lock:
        if key not in _engines:
            _engines[key] = Engine(torch.device("cuda", idx), map_mode)
        return _engines[key]


class KernelMap:
    """A built neighbour / gather map (``sc_kmap*``), freed with the object."""

    def __init__(self, engine, ptr, kind, n_in=None, n_out=None, kernel_volume=None, keepalive=None):
        self.engine = engine
        self.ptr = ptr
        self.kind = kind
        self._keepalive = keepalive
        if n_in is None or n_out is None or kernel_volume is None:
            info = self.info()  # waits for the build
            n_in, n_out, kernel_volume = info["n_in"], info["n_out"], info["kernel_volume"]
        self.n_in = int(n_in)
        self.n_out = int(n_out)
        self.kernel_volume = int(kernel_volume)

    def info(self):
        inf = L.ScKmapInfo()
        self.engine.check(self.engine.lib.sc_kmap_get_info(self.engine.handle, self.ptr, ctypes.byref(inf)),
                          "sc_kmap_get_info")
        return {k: getattr(inf, k) for k, _ in L.ScKmapInfo._fields_}

    def check(self):
        self.engine.check(self.engine.lib.sc_kmap_check(self.engine.handle, self.ptr), "sc_kmap_check")

    def export(self):
        """Canonical ``[n_out, K]`` int32 map on the device."""
        out = torch.empty((self.n_out, self.kernel_volume), dtype=torch.int32, device=self.engine.device)
        self.engine.bind_stream()
        self.engine.check(self.engine.lib.sc_kmap_export(self.engine.handle, self.ptr, _ptr(out)), "sc_kmap_export")
        return out

    def out_coords(self):
        """Parent coords of a down-sample map, ``[n_out, 4]`` int32."""
        out = torch.empty((self.n_out, 4), dtype=torch.int32, device=self.engine.device)
        self.engine.bind_stream()
        self.engine.check(self.engine.lib.sc_kmap_out_coords(self.engine.handle, self.ptr, _ptr(out)),
                          "sc_kmap_out_coords")
        return out

    def free(self):
        if self.ptr is not None and self.engine.handle:
            self.engine.bind_stream()
            self.engine.lib.sc_kmap_free(self.engine.handle, self.ptr)
        self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _coords_arg(coords):
    if coords.dtype != torch.int32 or coords.dim() != 2 or coords.shape[1] != 4:
        raise ValueError("coords must be an (N, 4) int32 tensor [b, x, y, z]")
    if not coords.is_cuda:
        raise ValueError("coords must be on a CUDA device")
    return coords.contiguous()


def _flags(tile_sort, check, halo=False):
    f = 0 if tile_sort else L.SC_BUILD_NO_TILE_SORT
    if halo:
        f |= L.SC_BUILD_HALO
    return f if check else f | L.SC_BUILD_DEFER_CHECK


def build_kmap(coords, dilation=1, engine=None, tile_sort=True, check=True, n_out=None, out_begin=0, halo=False):
    """Submanifold 3x3x3 neighbour map (``sc_kmap_build``).

    ``dilation`` is one int or ``(dil_x, dil_y, dil_z)`` -- the reference's
    ``(dilD, dilH, dilW)``, kd pairing with x (``sc_kmap_build_dilated``).

    With ``n_out`` / ``out_begin`` only rows ``[out_begin, out_begin + n_out)``
    are outputs (map row j is input row ``out_begin + j``) while neighbours are
    looked up among all rows (``sc_kmap_build_range``; sharded convs order a
    rank's owned voxels interior first, then boundary, then its halo).

    ``halo=True`` (``SC_BUILD_HALO``) keeps tiles in row order and adds per-tile
    halo lists, which lets bf16/f16 convs with Ci a multiple of 64 and Co <= 128
    run the halo-staged kernel; it suits spatially ordered rows (Morton or
    lexicographic).  The results equal those of the default map bit for bit.
    """
    coords = _coords_arg(coords)
    eng = engine or get_engine(coords.device)
    eng.bind_stream()
    p = ctypes.c_void_p()
    n = coords.shape[0]
    dil = tuple(int(d) for d in dilation) if hasattr(dilation, "__len__") else (int(dilation),) * 3
    if len(dil) != 3:
        raise ValueError("dilation must be an int or (dil_x, dil_y, dil_z)")
    if len(set(dil)) != 1:
        begin = int(out_begin)
        n_out = n - begin if n_out is None else int(n_out)
        eng.check(eng.lib.sc_kmap_build_dilated(eng.handle, _ptr(coords), n, begin, begin + n_out, dil[0], dil[1],
                                                dil[2], _flags(tile_sort, check, halo), ctypes.byref(p)),
                  "sc_kmap_build_dilated")
        return KernelMap(eng, p, L.SC_KMAP_SUBM, n, n_out, 27)
    dilation = dil[0]
    if n_out is None and out_begin == 0:
        eng.check(eng.lib.sc_kmap_build(eng.handle, _ptr(coords), n, 3, int(dilation),
                                        _flags(tile_sort, check, halo), ctypes.byref(p)), "sc_kmap_build")
        n_out = n
    else:
        n_out = n - int(out_begin) if n_out is None else int(n_out)
        eng.check(eng.lib.sc_kmap_build_range(eng.handle, _ptr(coords), n, int(out_begin), int(out_begin) + n_out, 3,
                                              int(dilation), _flags(tile_sort, check, halo), ctypes.byref(p)),
                  "sc_kmap_build_range")
    return KernelMap(eng, p, L.SC_KMAP_SUBM, n, n_out, 27)


def concat_kmaps(first, second, check=True):
    """Map whose tiles are ``first``'s then ``second``'s (``sc_kmap_concat``).

    Both are submanifold maps over the same input rows; output j of ``second``
    becomes output ``first.n_out + j``.  A sharded conv concatenates the map of
    its interior outputs (which read no halo row) with that of its boundary
    outputs, so ``conv3d(..., halo_wait=...)`` runs the interior tiles while
    the halo exchange is in flight.
    """
    if first.kind != L.SC_KMAP_SUBM or second.kind != L.SC_KMAP_SUBM:
        raise ValueError("concat_kmaps needs two submanifold maps")
    if first.engine is not second.engine or first.n_in != second.n_in:
        raise ValueError("concat_kmaps needs maps of one engine over the same input rows")
    eng = first.engine
    eng.bind_stream()
    p = ctypes.c_void_p()
    eng.check(eng.lib.sc_kmap_concat(eng.handle, first.ptr, second.ptr, _flags(True, check),
                                     ctypes.byref(p)), "sc_kmap_concat")
    return KernelMap(eng, p, L.SC_KMAP_SUBM, first.n_in, first.n_out + second.n_out, first.kernel_volume)


class HaloWait(collections.namedtuple("HaloWait", "flags world rank epoch")):
    """A halo exchange a conv waits for on the device: word r of the flag array
    at device address ``flags`` must reach ``epoch`` for every r != rank."""


def build_down2(coords, engine=None, tile_sort=True):
    """Stride-2 2x2x2 down-sample map (``sc_kmap_build_down2``)."""
    coords = _coords_arg(coords)
    eng = engine or get_engine(coords.device)
    eng.bind_stream()
    p = ctypes.c_void_p()
    eng.check(eng.lib.sc_kmap_build_down2(eng.handle, _ptr(coords), coords.shape[0], _flags(tile_sort, True),
                                          ctypes.byref(p)), "sc_kmap_build_down2")
    return KernelMap(eng, p, L.SC_KMAP_DOWN2)


def build_up2(down, tile_sort=True):
    """Transposed map of a down-sample map (``sc_kmap_build_up2``)."""
    eng = down.engine
    eng.bind_stream()
    p = ctypes.c_void_p()
    eng.check(eng.lib.sc_kmap_build_up2(eng.handle, down.ptr, _flags(tile_sort, True), ctypes.byref(p)),
              "sc_kmap_build_up2")
    return KernelMap(eng, p, L.SC_KMAP_UP2, down.n_out, down.n_in, 8, keepalive=down)


def conv3d(kmap, feats, weight, bias=None, residual=None, silu=False, layernorm=False, eps=1e-6, out=None,
           halo_wait=None):
    """``out = epilogue(bias + sum_v W[:, v] . feats[map[:, v]])`` through ``sc_conv3d``.

    With ``halo_wait`` (a :class:`HaloWait`) the conv waits on the device for
    that halo exchange before it gathers halo rows (``sc_conv3d_halo``).
    """
    dt = _DTYPES.get(feats.dtype)
    if dt is None:
        raise TypeError(f"unsupported feature dtype {feats.dtype}")
    co, ci = int(weight.shape[0]), int(weight.shape[-1])
    if weight.numel() != co * ci * kmap.kernel_volume:
        raise ValueError(f"weight {tuple(weight.shape)} does not match a {kmap.kernel_volume}-offset kernel")
    if feats.shape != (kmap.n_in, ci):
        raise ValueError(f"feats {tuple(feats.shape)} != ({kmap.n_in}, {ci})")
    feats = feats.contiguous()
    weight = weight.to(feats.dtype).contiguous()
    if bias is not None:
        bias = bias.to(feats.dtype).contiguous()
    if residual is not None:
        residual = residual.to(feats.dtype).contiguous()
        if residual.shape != (kmap.n_out, co):
            raise ValueError("residual must be (n_out, Co)")
    if out is None:
        out = torch.empty((kmap.n_out, co), dtype=feats.dtype, device=feats.device)
    epi = (L.SC_EPI_SILU if silu else 0) | (L.SC_EPI_RESIDUAL if residual is not None else 0) | \
          (L.SC_EPI_LAYERNORM if layernorm else 0)
    eng = kmap.engine
    eng.bind_stream()
    if halo_wait is None:
        eng.check(eng.lib.sc_conv3d(eng.handle, kmap.ptr, _ptr(feats), _ptr(weight), _ptr(bias), _ptr(residual),
                                    _ptr(out), ci, co, dt, epi, float(eps)), "sc_conv3d")
    else:
        hw = halo_wait
        eng.check(eng.lib.sc_conv3d_halo(eng.handle, kmap.ptr, _ptr(feats), _ptr(weight), _ptr(bias),
                                         _ptr(residual), _ptr(out), ci, co, dt, epi, float(eps),
                                         ctypes.c_void_p(int(hw.flags)), int(hw.world), int(hw.rank),
                                         int(hw.epoch) & 0xFFFFFFFF), "sc_conv3d_halo")
    return out


def layernorm_silu(x, silu=True, eps=1e-6, engine=None):
    """In-place row LayerNorm (no affine) + optional SiLU."""
    eng = engine or get_engine(x.device)
    eng.bind_stream()
    eng.check(eng.lib.sc_layernorm_silu(eng.handle, _ptr(x), x.shape[0], x.shape[1], _DTYPES[x.dtype],
                                        1 if silu else 0, float(eps)), "sc_layernorm_silu")
    return x


class SparseTensor:
    """Sparse voxels: coords ``(N, 4)`` int32 ``[b, x, y, z]`` + feats ``(N, C)``.

    Mirrors ``src/sparse/sparse_tensor.ts:18-121``: the spatial cache is a dict
    keyed by scale and shared by ``replace()``, so every conv on the same
    coords reuses one neighbour map.
    """

    def __init__(self, feats, coords, shape=None, scale=(1, 1, 1), cache=None):
        self.feats = feats
        self.coords = coords
        self._shape = shape
        self._scale = tuple(scale)
        self._spatial_cache = {} if cache is None else cache

    @property
    def scale(self):
        return self._scale

    @property
    def device(self):
        return self.feats.device

    @property
    def dtype(self):
        return self.feats.dtype

    def get_spatial_cache(self, key):
        return self._spatial_cache.get(self._scale, {}).get(key)

    def register_spatial_cache(self, key, value):
        self._spatial_cache.setdefault(self._scale, {})[key] = value

    def clear_spatial_cache(self):
        self._spatial_cache.clear()

    def replace(self, feats, coords=None):
        if coords is None:
            return SparseTensor(feats, self.coords, self._shape, self._scale, self._spatial_cache)
        return SparseTensor(feats, coords, None, self._scale, None)

    @property
    def spatial_shape(self):
        s = self.get_spatial_cache("shape")
        if s is None:
            s = tuple(int(v) + 1 for v in self.coords[:, 1:].amax(0).tolist()) if self.coords.shape[0] else (0, 0, 0)
            self.register_spatial_cache("shape", s)
        return s

    def __repr__(self):
        return f"SparseTensor(voxels={self.feats.shape[0]}, channels={self.feats.shape[1]}, dtype={self.dtype})"


class SparseConv3d:
    """Submanifold sparse conv (3x3x3), the drop-in for ``SparseConv3d`` of
    ``src/sparse/ops/conv3d.ts:18-222``.

    ``weight``: ``(Co, 3, 3, 3, Ci)``; ``bias``: ``(Co,)`` or None.
    """

    def __init__(self, weight, bias=None, kernel_size=(3, 3, 3), dilation=(1, 1, 1)):
        ks = tuple(kernel_size) if not isinstance(kernel_size, int) else (kernel_size,) * 3
        dl = tuple(dilation) if not isinstance(dilation, int) else (dilation,) * 3
        if ks != (3, 3, 3):
            raise NotImplementedError("only 3x3x3 submanifold kernels are implemented")
        if weight.dim() != 5 or tuple(weight.shape[1:4]) != ks:
            raise ValueError("weight must be (Co, Kd, Kh, Kw, Ci)")
        self.weight = weight
        self.bias = bias
        self.kernel_size = ks
        self.dilation = dl

    @property
    def V(self):
        return self.kernel_size[0] * self.kernel_size[1] * self.kernel_size[2]

    def cache_key(self):
        kd, kh, kw = self.kernel_size
        dd, dh, dw = self.dilation
        return f"conv_neighbors_{kw}x{kh}x{kd}_dil{dw}x{dh}x{dd}"

    def neighbour_map(self, x):
        km = x.get_spatial_cache(self.cache_key())
        if km is None:
            km = build_kmap(x.coords, self.dilation)
            x.register_spatial_cache(self.cache_key(), km)
        return km

    def forward(self, x, silu=False, residual=None):
        if not x.feats.is_cuda:
            raise ValueError("SparseConv3d requires GPU input")
        km = self.neighbour_map(x)
        out = conv3d(km, x.feats, self.weight, self.bias, residual=residual, silu=silu)
        return x.replace(out)

    __call__ = forward


class SparseConvDown2:
    """Stride-2 2x2x2 sparse conv: ``weight (Co, 2, 2, 2, Ci)``.

    Output coords are the unique ``(b, x>>1, y>>1, z>>1)`` in ascending
    lexicographic order.  The down map is cached on the input's spatial cache
    and handed to the output so that ``SparseConvUp2`` can return to the fine
    coords.
    """

    def __init__(self, weight, bias=None):
        if weight.dim() != 5 or tuple(weight.shape[1:4]) != (2, 2, 2):
            raise ValueError("weight must be (Co, 2, 2, 2, Ci)")
        self.weight = weight
        self.bias = bias

    def forward(self, x, silu=False):
        km = x.get_spatial_cache("down2_map")
        if km is None:
            km = build_down2(x.coords)
            x.register_spatial_cache("down2_map", km)
        out = conv3d(km, x.feats, self.weight, self.bias, silu=silu)
        coarse = SparseTensor(out, km.out_coords(), None, tuple(2 * s for s in x.scale))
        coarse.register_spatial_cache("up2_source", (km, x))
        return coarse

    __call__ = forward


class SparseConvUp2:
    """Transposed 2x2x2 sparse conv back onto the fine coords of the matching
    ``SparseConvDown2`` input: ``out[c] = bias + W[:, slot(c), :] . g[parent(c)]``."""

    def __init__(self, weight, bias=None):
        if weight.dim() != 5 or tuple(weight.shape[1:4]) != (2, 2, 2):
            raise ValueError("weight must be (Co, 2, 2, 2, Ci)")
        self.weight = weight
        self.bias = bias

    def forward(self, x, silu=False):
        src = x.get_spatial_cache("up2_source")
        if src is None:
            raise ValueError("SparseConvUp2 needs a tensor produced by SparseConvDown2")
        down, fine = src
        km = fine.get_spatial_cache("up2_map")
        if km is None:
            km = build_up2(down)
            fine.register_spatial_cache("up2_map", km)
        out = conv3d(km, x.feats, self.weight, self.bias, silu=silu)
        return fine.replace(out)

    __call__ = forward


def sparse_conv3d_forward(feats, coords, weight, bias=None, dilation=1, kmap=None):
    """Function-level submanifold conv for a ``SPARSE_CONV_BACKEND`` module.

    Returns ``(out, kmap)``; pass ``kmap`` back in to reuse the neighbour map
    for later layers on the same coords.
    """
    if kmap is None:
        kmap = build_kmap(coords, dilation)
    return conv3d(kmap, feats, weight, bias), kmap


def sparse_resblock(x, w1, b1, w2, b2, eps=1e-6):
    """conv -> LayerNorm -> SiLU -> conv + identity skip; both convs share one map
    and the LN/SiLU and the skip add are fused into the conv epilogues."""
    km = SparseConv3d(w1).neighbour_map(x)
    h = conv3d(km, x.feats, w1, b1, silu=True, layernorm=True, eps=eps)
    out = conv3d(km, h, w2, b2, residual=x.feats)
    return x.replace(out)


def conv3d_depthwise(kmap, feats, weight, bias=None, out=None):
    """Depthwise 3x3x3 submanifold conv (``sc_conv3d_depthwise``):
    ``out[n, c] = bias[c] + sum_v W[c, v] * feats[map[n, v], c]``.

    ``weight`` is ``(C, 3, 3, 3, 1)`` (or ``(C, 27)``); C a multiple of 8."""
    dt = _DTYPES.get(feats.dtype)
    if dt is None:
        raise TypeError(f"unsupported feature dtype {feats.dtype}")
    if kmap.kind != L.SC_KMAP_SUBM or kmap.kernel_volume != 27:
        raise ValueError("depthwise conv needs a 3x3x3 submanifold map")
    c = int(feats.shape[1]) if feats.dim() == 2 else -1
    if feats.shape != (kmap.n_in, c) or weight.numel() != 27 * c:
        raise ValueError(f"feats {tuple(feats.shape)} / weight {tuple(weight.shape)} do not match "
                         f"({kmap.n_in}, C) / (C, 3, 3, 3, 1)")
    feats = feats.contiguous()
    weight = weight.to(feats.dtype).contiguous()
    if bias is not None:
        bias = bias.to(feats.dtype).contiguous()
    if out is None:
        out = torch.empty((kmap.n_out, c), dtype=feats.dtype, device=feats.device)
    eng = kmap.engine
    eng.bind_stream()
    eng.check(eng.lib.sc_conv3d_depthwise(eng.handle, kmap.ptr, _ptr(feats), _ptr(weight), _ptr(bias), _ptr(out),
                                          c, dt), "sc_conv3d_depthwise")
    return out


def _linear(x, weight, bias, layout):
    w = weight.to(x.dtype)
    w = w.t() if layout == "out_in" else w
    if bias is None:
        return x @ w
    return torch.addmm(bias.to(x.dtype), x, w)


def sparse_convnext_block(x, dw_weight, dw_bias, l0_weight, l0_bias, l2_weight, l2_bias, eps=1e-6,
                          linear_layout="out_in"):
    """The sparse VAE decoder's ConvNeXt block
    (``src/models/sparse_unet_vae_decoder.ts:48-77``): ``dw_conv`` ->
    LayerNorm -> Linear0 -> LayerNorm -> SiLU -> Linear2, plus identity skip.

    * ``dw_weight`` ``(C, 3, 3, 3, C)``: a full conv with the LayerNorm fused
      into its epilogue (``sc_conv3d`` with ``SC_EPI_LAYERNORM``), the way the
      TS runs it (``src/sparse/ops/conv3d.ts:48``);
    * ``dw_weight`` ``(C, 3, 3, 3, 1)``: the depthwise conv
      (``sc_conv3d_depthwise``) followed by the engine's row LayerNorm;
    * ``dw_weight`` None: LayerNorm of ``x.feats`` (the TS's ``dwConv`` null).

    Both Linears are plain cuBLAS GEMMs (``torch.addmm``); the LayerNorm + SiLU
    between them is the engine's row kernel.  ``linear_layout`` "out_in"
    takes ``torch.nn.Linear`` weights ``(out, in)``; "in_out" takes the
    ``(in, out)`` matrices the TS ``matmul(a, b)`` multiplies by
    (``src/runtime/ops/matmul.ts:16-26``)."""
    if linear_layout not in ("out_in", "in_out"):
        raise ValueError("linear_layout must be 'out_in' or 'in_out'")
    if not x.feats.is_cuda:
        raise ValueError("sparse_convnext_block runs on CUDA tensors only")
    f = x.feats.contiguous()
    c = int(f.shape[1])
    if dw_weight is None:
        h = layernorm_silu(f.clone(), silu=False, eps=eps)
    else:
        km = SparseConv3d(dw_weight).neighbour_map(x)
        if dw_weight.shape[-1] == 1 and c != 1:
            h = layernorm_silu(conv3d_depthwise(km, f, dw_weight, dw_bias), silu=False, eps=eps)
        else:
            h = conv3d(km, f, dw_weight, dw_bias, layernorm=True, eps=eps)
    h = layernorm_silu(_linear(h, l0_weight, l0_bias, linear_layout).contiguous(), silu=True, eps=eps)
    out = _linear(h, l2_weight, l2_bias, linear_layout)
    return x.replace(out.add_(f))


def subdivide2(x, child_mask=None):
    """2x2x2 subdivision of a :class:`SparseTensor` (``sc_subdivide2``).

    Every voxel ``(b, x, y, z)`` becomes ``(b, 2x+i, 2y+j, 2z+k)``, child
    ``s = i*4 + j*2 + k``, in (voxel, s) order, each with a copy of its
    voxel's features.  ``child_mask`` keeps only some children: an ``(N, 8)``
    bool tensor, or ``(N,)`` uint8 with bit s for child s (the subdivision
    logits of ``SparseResBlockUpsample3d`` thresholded at 0 give it).  The
    result's scale is halved and its spatial cache is new.  Returns
    ``(fine, parent)`` with ``parent[j]`` the voxel row of child j."""
    coords = _coords_arg(x.coords)
    n = int(coords.shape[0])
    feats = x.feats.contiguous()
    eng = get_engine(coords.device)
    mask = None
    if child_mask is not None:
        m = child_mask.to(coords.device)
        if m.dtype == torch.bool:
            if m.shape != (n, 8):
                raise ValueError("a bool child_mask must be (N, 8)")
            bits = torch.tensor([1, 2, 4, 8, 16, 32, 64, 128], dtype=torch.int32, device=m.device)
            m = (m.to(torch.int32) * bits).sum(1).to(torch.uint8)
        elif m.dtype != torch.uint8 or m.shape != (n,):
            raise ValueError("child_mask must be (N, 8) bool or (N,) uint8")
        mask = m.contiguous()
    row_bytes = int(feats.shape[1]) * feats.element_size()
    if row_bytes % 16 != 0:
        raise ValueError("feature rows must be a multiple of 16 bytes")
    eng.bind_stream()
    cnt = ctypes.c_int64()
    if mask is None:
        total = 8 * n
    else:
        eng.check(eng.lib.sc_subdivide2(eng.handle, _ptr(coords), n, _ptr(mask), None, 0, None, None, None, 0,
                                        ctypes.byref(cnt)), "sc_subdivide2")
        total = int(cnt.value)
    out_c = torch.empty((total, 4), dtype=torch.int32, device=coords.device)
    parent = torch.empty(total, dtype=torch.int32, device=coords.device)
    out_f = torch.empty((total, feats.shape[1]), dtype=feats.dtype, device=feats.device)
    eng.check(eng.lib.sc_subdivide2(eng.handle, _ptr(coords), n, _ptr(mask), _ptr(feats), row_bytes, _ptr(out_c),
                                    _ptr(parent), _ptr(out_f), total, ctypes.byref(cnt)), "sc_subdivide2")
    return SparseTensor(out_f, out_c, None, tuple(s / 2 for s in x.scale)), parent


def sparse_attention(q, k, v, cu_seqlens_q, cu_seqlens_kv=None, scale=None, out=None):
    """Variable-length scaled dot-product attention (``sc_attention_varlen``),
    the ``sparseAttention`` of ``src/sparse/ops/attention.ts:14-80``.

    ``q`` ``(total_N, H, 64)``, ``k`` / ``v`` ``(total_N_kv, H, 64)`` (bf16 or
    f16, CUDA); ``cu_seqlens_q`` / ``cu_seqlens_kv`` the ``B + 1`` sequence
    offsets (any int sequence or tensor; read on the host, as the reference's
    ``Uint32Array`` are); ``cu_seqlens_kv`` defaults to ``cu_seqlens_q`` (self
    attention).  ``scale`` defaults to ``1 / sqrt(64)``.  Returns ``(total_N,
    H, 64)``; query rows of a sequence with no key rows are zero."""
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError("sparse_attention takes bf16 or f16 tensors")
    if not q.is_cuda:
        raise ValueError("sparse_attention runs on CUDA tensors only")
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3 or k.shape != v.shape or q.shape[1:] != k.shape[1:]:
        raise ValueError("q must be (N, H, D) and k, v (N_kv, H, D) with the same H and D")
    cu_q = torch.as_tensor(cu_seqlens_q, dtype=torch.int32).cpu().contiguous()
    cu_kv = cu_q if cu_seqlens_kv is None else torch.as_tensor(cu_seqlens_kv, dtype=torch.int32).cpu().contiguous()
    if cu_q.dim() != 1 or cu_kv.shape != cu_q.shape or cu_q.numel() < 2:
        raise ValueError("cu_seqlens must be 1-D with batch + 1 entries, the same count for q and kv")
    if int(cu_q[-1]) != q.shape[0] or int(cu_kv[-1]) != k.shape[0]:
        raise ValueError("cu_seqlens must end at the token counts of q and k/v")
    heads, d = int(q.shape[1]), int(q.shape[2])
    q, k, v = q.contiguous(), k.to(q.dtype).contiguous(), v.to(q.dtype).contiguous()
    if out is None:
        out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    eng = get_engine(q.device)
    eng.bind_stream()
    eng.check(eng.lib.sc_attention_varlen(eng.handle, _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                          ctypes.c_void_p(cu_q.data_ptr()), ctypes.c_void_p(cu_kv.data_ptr()),
                                          cu_q.numel() - 1, heads, d, scale, _DTYPES[q.dtype]),
              "sc_attention_varlen")
    return out
