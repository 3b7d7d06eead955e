"""Host-to-host sparse conv with the transfers of consecutive calls overlapped.

A serving loop that receives voxel sets in host memory and returns features to
host memory spends most of each call on PCIe: on the 256^3 shell workload one
call moves 110 MB in (coords + bf16 feats) and 104 MB out, about 2 ms each way,
against 0.7 ms of map build + conv on the GPU.  ``HostConvPipeline`` keeps
``depth`` slots of device buffers and three streams so that call k+1's
host-to-device copy, call k's map build + conv and call k-1's device-to-host
copy run at the same time; every call still performs its own copies.  With
``depth`` slots, call k's input copy starts once call k-depth has finished, so
the period per call is max(H2D, (H2D + compute + D2H) / depth); the default of
3 slots lets the input copy run back to back on the 256^3 workload.

    pipe = HostConvPipeline(weight, bias)          # weight (Co, 3, 3, 3, Ci) on the GPU
    for coords_h, feats_h, out_h in batches:        # pinned host tensors
        pipe.submit(coords_h, feats_h, out_h)       # returns at once
    pipe.synchronize()                              # all outputs written, errors raised

A slot is reused only after the host has seen its previous call finish, at
which point that call's neighbour-map status is checked and its map freed, so
a duplicate or out-of-range coordinate raises from the ``submit`` that reuses
the slot (or from ``synchronize``) instead of from the call that carried it.
"""
from __future__ import annotations

import torch

from .sparse_conv import build_kmap, conv3d, get_engine

__all__ = ["HostConvPipeline"]


class _Slot:
    def __init__(self):
        self.coords = None
        self.feats = None
        self.out = None
        self.kmap = None
        self.done = None  # event after the device-to-host copy of the slot's last call


class HostConvPipeline:
    """``depth``-slot pipeline of submanifold convs from pinned host inputs to pinned host outputs."""

    def __init__(self, weight, bias=None, dilation=1, depth=3, engine=None):
        if not weight.is_cuda:
            raise ValueError("weight must be on a CUDA device (layer parameters stay resident)")
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.device = weight.device
        self.weight = weight
        self.bias = bias
        self.dilation = int(dilation)
        self.engine = engine or get_engine(self.device)
        self.s_in = torch.cuda.Stream(self.device)
        self.s_comp = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)
        self.s_status = torch.cuda.Stream(self.device)
        self.slots = [_Slot() for _ in range(depth)]
        self.calls = 0

    def _retire(self, slot):
        """Waits for the slot's last call, checks its map status and frees the map."""
        if slot.done is not None:
            slot.done.synchronize()
            slot.done = None
        if slot.kmap is not None:
            km, slot.kmap = slot.kmap, None
            with torch.cuda.stream(self.s_status):
                self.engine.bind_stream(self.s_status)
                km.check()
                km.free()

    def _reserve(self, slot, n, ci, co, dtype):
        if slot.coords is None or slot.coords.shape[0] < n:
            cap = max(n, 1)
            slot.coords = torch.empty((cap, 4), dtype=torch.int32, device=self.device)
        if slot.feats is None or slot.feats.shape[0] < n or slot.feats.shape[1] != ci or slot.feats.dtype != dtype:
            slot.feats = torch.empty((max(n, 1), ci), dtype=dtype, device=self.device)
        if slot.out is None or slot.out.shape[0] < n or slot.out.shape[1] != co or slot.out.dtype != dtype:
            slot.out = torch.empty((max(n, 1), co), dtype=dtype, device=self.device)

    def submit(self, coords_h, feats_h, out_h):
        """Enqueues one conv: ``coords_h`` (N, 4) int32, ``feats_h`` (N, Ci) and ``out_h`` (N, Co),
        all in pinned host memory.  ``out_h`` is written when ``synchronize`` returns."""
        n = int(coords_h.shape[0])
        ci, co = int(feats_h.shape[1]), int(self.weight.shape[0])
        if coords_h.is_cuda or feats_h.is_cuda or out_h.is_cuda:
            raise ValueError("HostConvPipeline takes host tensors; use sparse_conv3d_forward for device tensors")
        if feats_h.shape[0] != n or tuple(out_h.shape) != (n, co) or out_h.dtype != feats_h.dtype:
            raise ValueError("feats_h must be (N, Ci) and out_h (N, Co) of the same dtype")
        slot = self.slots[self.calls % len(self.slots)]
        self.calls += 1
        self._retire(slot)
        if n == 0:
            return
        self._reserve(slot, n, ci, co, feats_h.dtype)
        c_d, f_d, o_d = slot.coords[:n], slot.feats[:n], slot.out[:n]
        with torch.cuda.stream(self.s_in):
            c_d.copy_(coords_h, non_blocking=True)
            f_d.copy_(feats_h, non_blocking=True)
            ev_in = torch.cuda.Event()
            ev_in.record(self.s_in)
        with torch.cuda.stream(self.s_comp):
            self.s_comp.wait_event(ev_in)
            km = build_kmap(c_d, self.dilation, engine=self.engine, check=False)
            conv3d(km, f_d, self.weight, self.bias, out=o_d)
            ev_comp = torch.cuda.Event()
            ev_comp.record(self.s_comp)
        with torch.cuda.stream(self.s_out):
            self.s_out.wait_event(ev_comp)
            out_h.copy_(o_d, non_blocking=True)
            done = torch.cuda.Event()
            done.record(self.s_out)
        slot.kmap = km
        slot.done = done

    def synchronize(self):
        """Waits for every submitted call and raises the first map or conv error."""
        for slot in self.slots:
            self._retire(slot)
        self.engine.bind_stream(self.s_status)
        self.engine.synchronize()
