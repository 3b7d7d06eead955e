"""B200-native (sm_100a) submanifold sparse conv3d engine for TRELLIS.2.

A drop-in for the reference sparse-conv operator (``SparseConv3d`` of
``src/sparse/ops/conv3d.ts`` / the ``SPARSE_CONV_BACKEND`` module of
``trellis2/modules/sparse/conv``): kernel-map construction (hash or one-sweep
radix sort), a tcgen05 implicit-GEMM conv fed by TMA row gathers and TMA
weight tiles, a depthwise conv, 2x2x2 subdivision, varlen attention, stride-2 down/up convs, Morton-range sharding across GPUs, and a
host-to-host pipeline that overlaps the transfers of consecutive calls.  All compute is in
``libsparseconv_b200.so`` (C ABI in ``include/sparse_conv_b200.h``).
"""
from . import _lib
from ._lib import SparseConvError, DuplicateCoordError, CoordRangeError
from .sparse_conv import (
    Engine, get_engine, KernelMap, build_kmap, concat_kmaps, HaloWait, build_down2, build_up2, conv3d, layernorm_silu,
    SparseTensor, SparseConv3d, SparseConvDown2, SparseConvUp2, sparse_conv3d_forward, sparse_resblock,
    conv3d_depthwise, sparse_convnext_block, subdivide2, sparse_attention,
)
from . import coords_io
from .host_pipeline import HostConvPipeline
from . import workloads
from . import conv_b200

__version__ = "0.1.0"
