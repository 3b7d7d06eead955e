"""``SPARSE_CONV_BACKEND=b200``: the sparse-conv modules of ``trellis2/modules/sparse/conv`` on this engine.

The reference selects its sparse-conv implementation with the
``SPARSE_CONV_BACKEND`` environment variable (``README.md:27,109``; set by its
callers at ``trellis_webgpu.ts:66,99`` and ``src/pipeline/run.ts:179``); the
backend it runs on AMD is ``conv_none.py``.  This module is the ``b200``
choice: ``torch.nn`` modules holding the checkpoint weight layout
``(Co, Kd, Kh, Kw, Ci)`` (``src/sparse/ops/conv3d.ts:5,19,48-49``) that run
every conv on the CUDA library.

* ``SparseConv3d(in_channels, out_channels, kernel_size, stride=1, dilation=1,
  padding=None, bias=True, indice_key=None)``: stride 1 with a 3x3x3 kernel is
  the submanifold conv (neighbour map cached on the input tensor under the
  reference's key ``conv_neighbors_{Kw}x{Kh}x{Kd}_dil..``,
  ``src/sparse/ops/conv3d.ts:63-72``); stride 2 with a 2x2x2 kernel is the
  stride-2 down-sample (parents ``(b, x>>1, y>>1, z>>1)``).
* ``SparseInverseConv3d(in_channels, out_channels, kernel_size=2, stride=2,
  ...)``: the transposed 2x2x2 conv back onto the fine coords of the tensor a
  ``SparseConv3d`` down-sampled.
* ``sparse_conv3d_forward(feats, coords, weight, bias, dilation, kmap)``: the
  function-level entry.

The upstream module's exact constructor signature is not in the reference
tree (its ``trellis2`` package is an empty submodule); the arguments above are
the ones its callers pass in the TRELLIS family of models, and arguments this
engine does not need (``padding``, ``indice_key``) are accepted and ignored.
Inputs are any sparse tensor with ``feats``, ``coords``, ``replace`` and the
spatial-cache methods (this package's ``SparseTensor`` has them).  There is no
CPU path: CPU inputs raise ``ValueError``.
"""
from __future__ import annotations

import math
import os

import torch
from torch import nn

from .sparse_conv import SparseTensor, build_down2, build_kmap, build_up2, conv3d, sparse_conv3d_forward

__all__ = ["BACKEND_NAME", "SparseConv3d", "SparseInverseConv3d", "sparse_conv3d_forward", "load_backend",
           "SparseTensor"]

BACKEND_NAME = "b200"


def load_backend(name=None):
    """The backend module ``SPARSE_CONV_BACKEND`` (or ``name``) selects: this module for ``b200``."""
    name = os.environ.get("SPARSE_CONV_BACKEND", BACKEND_NAME) if name is None else name
    if name != BACKEND_NAME:
        raise ValueError(f"SPARSE_CONV_BACKEND={name!r}: this package provides only {BACKEND_NAME!r}")
    import sys
    return sys.modules[__name__]


def _triple(v, what):
    t = tuple(int(x) for x in v) if hasattr(v, "__len__") else (int(v),) * 3
    if len(t) != 3:
        raise ValueError(f"{what} must be an int or a triple")
    return t


def _need_gpu(x):
    if not x.feats.is_cuda:
        raise ValueError("the b200 sparse-conv backend runs on CUDA tensors only")


class SparseConv3d(nn.Module):
    """Submanifold 3x3x3 conv (stride 1) or stride-2 2x2x2 down-sample conv."""

    def __init__(self, in_channels, out_channels, kernel_size=3, stride=1, dilation=1, padding=None, bias=True,
                 indice_key=None, device=None, dtype=None):
        super().__init__()
        self.kernel_size = _triple(kernel_size, "kernel_size")
        self.stride = _triple(stride, "stride")
        self.dilation = _triple(dilation, "dilation")
        if self.stride == (1, 1, 1):
            if self.kernel_size != (3, 3, 3):
                raise NotImplementedError("submanifold convs are implemented for 3x3x3 kernels")
        elif self.stride == (2, 2, 2):
            if self.kernel_size != (2, 2, 2) or self.dilation != (1, 1, 1):
                raise NotImplementedError("stride-2 convs are implemented for 2x2x2 kernels without dilation")
        else:
            raise NotImplementedError("stride must be 1 (submanifold) or 2 (down-sample)")
        self.in_channels, self.out_channels = int(in_channels), int(out_channels)
        self.weight = nn.Parameter(torch.empty((out_channels, *self.kernel_size, in_channels), device=device,
                                               dtype=dtype))
        self.bias = nn.Parameter(torch.empty(out_channels, device=device, dtype=dtype)) if bias else None
        self.reset_parameters()

    def reset_parameters(self):
        fan_in = self.in_channels * math.prod(self.kernel_size)
        nn.init.normal_(self.weight, 0.0, 1.0 / math.sqrt(fan_in))
        if self.bias is not None:
            nn.init.zeros_(self.bias)

    def cache_key(self):
        kd, kh, kw = self.kernel_size
        dd, dh, dw = self.dilation
        return f"conv_neighbors_{kw}x{kh}x{kd}_dil{dw}x{dh}x{dd}"

    def forward(self, x):
        _need_gpu(x)
        feats = x.feats
        w = self.weight.to(feats.dtype)
        b = None if self.bias is None else self.bias.to(feats.dtype)
        if self.stride == (1, 1, 1):
            km = x.get_spatial_cache(self.cache_key())
            if km is None:
                km = build_kmap(x.coords, self.dilation)
                x.register_spatial_cache(self.cache_key(), km)
            return x.replace(conv3d(km, feats, w, b))
        km = x.get_spatial_cache("down2_map")
        if km is None:
            km = build_down2(x.coords)
            x.register_spatial_cache("down2_map", km)
        out = conv3d(km, feats, w, b)
        scale = tuple(2 * s for s in getattr(x, "scale", (1, 1, 1)))
        coarse = SparseTensor(out, km.out_coords(), None, scale)
        coarse.register_spatial_cache("up2_source", (km, x))
        return coarse


class SparseInverseConv3d(nn.Module):
    """Transposed 2x2x2 conv (stride 2) back onto the fine coords of the
    tensor that a stride-2 ``SparseConv3d`` down-sampled."""

    def __init__(self, in_channels, out_channels, kernel_size=2, stride=2, dilation=1, bias=True, indice_key=None,
                 device=None, dtype=None):
        super().__init__()
        if _triple(kernel_size, "kernel_size") != (2, 2, 2) or _triple(stride, "stride") != (2, 2, 2):
            raise NotImplementedError("inverse convs are implemented for 2x2x2 kernels with stride 2")
        if _triple(dilation, "dilation") != (1, 1, 1):
            raise NotImplementedError("inverse convs take no dilation")
        self.in_channels, self.out_channels = int(in_channels), int(out_channels)
        self.weight = nn.Parameter(torch.empty((out_channels, 2, 2, 2, in_channels), device=device, dtype=dtype))
        self.bias = nn.Parameter(torch.empty(out_channels, device=device, dtype=dtype)) if bias else None
        nn.init.normal_(self.weight, 0.0, 1.0 / math.sqrt(8 * in_channels))
        if self.bias is not None:
            nn.init.zeros_(self.bias)

    def forward(self, x):
        _need_gpu(x)
        src = x.get_spatial_cache("up2_source")
        if src is None:
            raise ValueError("SparseInverseConv3d needs a tensor produced by a stride-2 SparseConv3d")
        down, fine = src
        km = fine.get_spatial_cache("up2_map")
        if km is None:
            km = build_up2(down)
            fine.register_spatial_cache("up2_map", km)
        feats = x.feats
        b = None if self.bias is None else self.bias.to(feats.dtype)
        return fine.replace(conv3d(km, feats, self.weight.to(feats.dtype), b))
