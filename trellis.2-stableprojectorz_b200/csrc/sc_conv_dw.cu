// Depthwise 3x3x3 submanifold conv: out[n, c] = bias[c] + sum_v W[c, v] *
// f[map[n, v], c], weight (C, 3, 3, 3, 1).
//
// This is the `dw_conv` of the sparse VAE decoder's ConvNeXt block
// (src/models/sparse_unet_vae_decoder.ts:48-59,122-132) when its checkpoint
// weight is depthwise; the TS port runs every conv as a dense Ci -> Co conv
// (src/sparse/ops/conv3d.ts:48), which for a depthwise weight would need
// Ci == 1.  Each output channel reads only its own input channel, so the op
// is a gather-bound elementwise sum: no tensor-core contraction.
//
// It walks the conv kernels' tile layout of the map: a block takes 32 rows of
// one 128-row tile and 64 channels (8 threads per row, 8 channels each), with
// the block's 27 x 64 weight slab in shared memory; per offset present in the
// tile each thread reads its row's gather index and 16 bytes (bf16/f16) or
// 32 bytes (f32) of the source row, and accumulates in f32 in ascending
// offset order, so results do not depend on the tile order.
#include "sc_common.cuh"
#include "sc_internal.h"

#include <algorithm>
#include <type_traits>

namespace sc {
namespace {

constexpr int kDwRows = 32;      // rows per block (a quarter tile)
constexpr int kDwChans = 64;     // channels per block
constexpr int kDwVec = 8;        // channels per thread
constexpr int kDwThreads = kDwRows * (kDwChans / kDwVec);  // 256
constexpr int kDwBlocksPerSm = 6;  // resident blocks at <= 40 registers a thread

template <typename T>
__device__ __forceinline__ void load8(const T* src, float (&x)[kDwVec]) {
  if constexpr (std::is_same_v<T, float>) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(src));
    const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  } else {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f;
      if constexpr (std::is_same_v<T, __nv_bfloat16>) f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
      else f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      x[2 * j] = f.x;
      x[2 * j + 1] = f.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* dst, const float (&x)[kDwVec]) {
  if constexpr (std::is_same_v<T, float>) {
    reinterpret_cast<float4*>(dst)[0] = make_float4(x[0], x[1], x[2], x[3]);
    reinterpret_cast<float4*>(dst)[1] = make_float4(x[4], x[5], x[6], x[7]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (std::is_same_v<T, __nv_bfloat16>) {
        const __nv_bfloat162 b = __floats2bfloat162_rn(x[2 * j], x[2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&b);
      } else {
        const __half2 b = __floats2half2_rn(x[2 * j], x[2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&b);
      }
    }
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}
template <typename T>
__device__ __forceinline__ float to_f32(T x) {
  if constexpr (std::is_same_v<T, float>) return x;
  else return static_cast<float>(x);
}

// acc[k] += W[v, 8*lc + k] * x[k] from the swizzled weight slab of offset v
// (sWv[half][lc][4], see k_conv_dw).
__device__ __forceinline__ void fma_w8(const float (*sWv)[kDwChans / kDwVec][4], int lc, const float (&x)[kDwVec],
                                       float (&acc)[kDwVec]) {
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const float4 w4 = *reinterpret_cast<const float4*>(sWv[hh][lc]);
    acc[4 * hh + 0] = fmaf(w4.x, x[4 * hh + 0], acc[4 * hh + 0]);
    acc[4 * hh + 1] = fmaf(w4.y, x[4 * hh + 1], acc[4 * hh + 1]);
    acc[4 * hh + 2] = fmaf(w4.z, x[4 * hh + 2], acc[4 * hh + 2]);
    acc[4 * hh + 3] = fmaf(w4.w, x[4 * hh + 3], acc[4 * hh + 3]);
  }
}

// Grid (tile blocks, channel blocks); each block strides over tiles, one
// quarter tile (32 rows x 64 channels) per pass.  The gather indices of a
// row's offsets are loaded together before its feature rows.
//
// Measured on B200 (406k voxels, 64 bf16 channels, L2 flushed): 123 us at
// six resident blocks per SM (40 registers, a few bytes spilled); 129 us at
// four (61 registers), 135 us at eight (32 registers, more spills).  The
// kernel is bound by load latency (long-scoreboard stalls) with the L1 data
// pipe about half busy.  Variants that were slower: whole tiles per
// block with the indices staged in shared memory and 9 predicated loads in
// flight per thread (223 us); the same batching in this layout (147 us);
// staging each tile's distinct source rows in shared memory from a
// SC_BUILD_HALO map (174-193 us, 1.6x the instructions).
template <typename T>
__global__ void __launch_bounds__(kDwThreads, kDwBlocksPerSm) k_conv_dw(const int32_t* __restrict__ gidx,
                                                        const int32_t* __restrict__ tile_rows,
                                                        const uint32_t* __restrict__ tile_mask, int64_t num_tiles,
                                                        const T* __restrict__ feats, const T* __restrict__ weight,
                                                        const T* __restrict__ bias, T* __restrict__ out, int c) {
  // Weights of offset v for channel c0 + 8*lc + k at sW[v][k / 4][lc][k % 4]:
  // a warp's 8 channel groups read one offset as two conflict-free 128-byte
  // float4 wavefronts (a plain [v][channel] layout costs 2-way conflicts on
  // every scalar read).
  __shared__ __align__(16) float sW[27][2][kDwChans / kDwVec][4];
  __shared__ __align__(16) float sB[kDwChans];
  const int c0 = blockIdx.y * kDwChans;
  const int nc = min(kDwChans, c - c0);
  for (int i = threadIdx.x; i < 27 * kDwChans; i += kDwThreads) {
    const int j = i / 27, v = i - j * 27;  // weight (C, 27): consecutive threads read consecutive offsets
    sW[v][(j & 7) >> 2][j >> 3][j & 3] = j < nc ? to_f32(weight[static_cast<int64_t>(c0 + j) * 27 + v]) : 0.f;
  }
  if (threadIdx.x < kDwChans)
    sB[threadIdx.x] = (bias && static_cast<int>(threadIdx.x) < nc) ? to_f32(bias[c0 + threadIdx.x]) : 0.f;
  __syncthreads();
  const int lc = threadIdx.x & 7;
  const int cc = lc * kDwVec;
  const int row = threadIdx.x >> 3;
  if (cc >= nc) return;
  const int64_t passes = num_tiles * (kTileRows / kDwRows);
  for (int64_t q = blockIdx.x; q < passes; q += gridDim.x) {
    const int64_t t = q >> 2;
    const int slot = static_cast<int>(q & 3) * kDwRows + row;
    const int r = tile_rows[t * kTileRows + slot];
    if (r < 0) continue;
    const uint32_t mask = tile_mask[t];
    int src[27];
#pragma unroll
    for (int v = 0; v < 27; ++v)
      src[v] = (mask >> v & 1u) ? __ldg(gidx + (t * 27 + v) * kTileRows + slot) : -1;
    float acc[kDwVec];
#pragma unroll
    for (int j = 0; j < kDwVec; ++j) acc[j] = 0.f;
#pragma unroll
    for (int v = 0; v < 27; ++v) {
      if (src[v] < 0) continue;
      float x[kDwVec];
      load8(feats + static_cast<int64_t>(src[v]) * c + c0 + cc, x);
      fma_w8(sW[v], lc, x, acc);
    }
#pragma unroll
    for (int j = 0; j < kDwVec; ++j) acc[j] += sB[cc + j];
    store8(out + static_cast<int64_t>(r) * c + c0 + cc, acc);
  }
}

template <typename T>
sc_status launch_dw(Handle* h, const KMap* km, const void* feats, const void* weight, const void* bias, void* out,
                    int c) {
  const int cblocks = (c + kDwChans - 1) / kDwChans;
  const int64_t passes = km->num_tiles * (kTileRows / kDwRows);
  // The grid fills every SM with resident blocks over all channel blocks.
  const int64_t want = std::max<int64_t>(1, (static_cast<int64_t>(h->num_sms) * kDwBlocksPerSm + cblocks - 1) / cblocks);
  const unsigned gx = static_cast<unsigned>(std::min<int64_t>(passes, want));
  ++h->launches;
  k_conv_dw<T><<<dim3(gx, cblocks), kDwThreads, 0, h->stream>>>(
      km->gidx, km->tile_rows, km->tile_mask, km->num_tiles, static_cast<const T*>(feats),
      static_cast<const T*>(weight), static_cast<const T*>(bias), static_cast<T*>(out), c);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SC_OK : cuda_error(h, e, "depthwise conv launch");
}

}  // namespace

sc_status conv_depthwise(Handle* h, const KMap* km, const void* feats, const void* weight, const void* bias,
                         void* out, int c, sc_dtype dtype) {
  if (km->n_out == 0 || km->num_tiles == 0) return SC_OK;
  if (h->debug_bounds) {
    const sc_status st = check_gather_bounds(h, km);
    if (st != SC_OK) return st;
  }
  switch (dtype) {
    case SC_F32: return launch_dw<float>(h, km, feats, weight, bias, out, c);
    case SC_BF16: return launch_dw<__nv_bfloat16>(h, km, feats, weight, bias, out, c);
    case SC_F16: return launch_dw<__half>(h, km, feats, weight, bias, out, c);
  }
  return set_error(h, SC_EINVAL, "unknown dtype");
}

}  // namespace sc
