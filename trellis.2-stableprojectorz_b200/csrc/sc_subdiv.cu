// 2x2x2 voxel subdivision: every voxel (b, x, y, z) becomes the children
// (b, 2x+i, 2y+j, 2z+k), child s = i*4 + j*2 + k, in (parent, s) order,
// optionally only the children whose bit s is set in a per-voxel byte mask,
// and each child row takes a copy of its parent's feature row.
//
// This is the upsample the TS decoder stands in for by doubling
// `spatialShape` while keeping the coords
// (src/models/sparse_unet_vae_decoder.ts:155-175); the subdividing module it
// replaces (TRELLIS SparseSubdivide and the subdivision mask predicted by
// SparseResBlockUpsample3d) is in the absent `trellis2` submodule.
//
// With a mask, child offsets come from an exclusive scan of popc(mask) over
// parents: per-block counts, a one-block scan of the block sums, then a
// block-local scan while writing.  Without one, parent p's children are rows
// 8p .. 8p+7 and nothing is counted.  Features are copied by a row gather
// in 16-byte vectors; the 8 children of a parent read its row back to back
// (from L1/L2), so DRAM sees about one read of the input rows.
#include "sc_common.cuh"
#include "sc_internal.h"

#include <algorithm>

namespace sc {
namespace {

constexpr int kSubBlock = 1024;  // parents per block of the count / write kernels

__device__ __forceinline__ uint32_t children(const uint8_t* mask, int64_t p) {
  return mask ? static_cast<uint32_t>(mask[p]) : 0xFFu;
}

__global__ void __launch_bounds__(kSubBlock) k_subdiv_count(const uint8_t* __restrict__ mask, int64_t n,
                                                            uint32_t* __restrict__ block_sums) {
  __shared__ uint32_t s[kSubBlock / 32];
  const int64_t p = blockIdx.x * static_cast<int64_t>(kSubBlock) + threadIdx.x;
  uint32_t c = p < n ? __popc(mask[p]) : 0u;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t t = s[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) block_sums[blockIdx.x] = t;
  }
}

// One block of 1024 threads: exclusive scan of the block sums in place (64-bit
// running total, so counts past 2^32 children are reported, not wrapped).
__global__ void __launch_bounds__(1024) k_subdiv_scan(uint32_t* block_sums, int64_t nb,
                                                      unsigned long long* total) {
  __shared__ uint32_t s[32];
  unsigned long long carry = 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t base = 0; base < nb; base += 1024) {
    const int64_t i = base + threadIdx.x;
    const uint32_t x = i < nb ? block_sums[i] : 0u;
    uint32_t incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      uint32_t w = s[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      s[lane] = w;  // inclusive warp totals
    }
    __syncthreads();
    const uint32_t warp_base = warp ? s[warp - 1] : 0u;
    // Block sums are at most 8 * 1024, so 1024 of them stay below 2^24; the
    // global offset is carried in 64 bits and written back truncated only
    // when the host has checked that the total fits.
    if (i < nb) block_sums[i] = static_cast<uint32_t>(carry) + warp_base + incl - x;
    const uint32_t chunk = s[31];
    __syncthreads();
    carry += chunk;
  }
  if (threadIdx.x == 0) *total = carry;
}

__global__ void __launch_bounds__(kSubBlock) k_subdiv_write(const int4* __restrict__ coords, int64_t n,
                                                            const uint8_t* __restrict__ mask,
                                                            const uint32_t* __restrict__ block_base,
                                                            int4* __restrict__ out_coords,
                                                            int32_t* __restrict__ out_parent) {
  __shared__ uint32_t s[kSubBlock / 32];
  const int64_t p = blockIdx.x * static_cast<int64_t>(kSubBlock) + threadIdx.x;
  const uint32_t m = p < n ? children(mask, p) : 0u;
  int64_t off;
  if (mask) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t c = __popc(m);
    uint32_t incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      uint32_t w = s[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      s[lane] = w;
    }
    __syncthreads();
    off = static_cast<int64_t>(block_base[blockIdx.x]) + (warp ? s[warp - 1] : 0u) + incl - c;
  } else {
    off = 8 * p;
  }
  if (p >= n) return;
  const int4 c = coords[p];
  uint32_t k = 0;
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {
    if (!(m >> ch & 1u)) continue;
    const int64_t j = off + k++;
    out_coords[j] = make_int4(c.x, 2 * c.y + (ch >> 2 & 1), 2 * c.z + (ch >> 1 & 1), 2 * c.w + (ch & 1));
    if (out_parent) out_parent[j] = static_cast<int32_t>(p);
  }
}

// out_feats[j] = feats[parent[j]], one thread per 16-byte vector.
__global__ void k_gather_rows(const uint4* __restrict__ feats, const int32_t* __restrict__ parent, int64_t rows,
                              int vecs, uint4* __restrict__ out) {
  const int64_t total = rows * vecs;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t j = e / vecs;
    const int v = static_cast<int>(e - j * vecs);
    out[e] = __ldg(feats + static_cast<int64_t>(__ldg(parent + j)) * vecs + v);
  }
}

}  // namespace

sc_status subdivide2(Handle* h, const int32_t* coords, int64_t n, const uint8_t* child_mask, const void* feats,
                     int row_bytes, int32_t* out_coords, int32_t* out_parent, void* out_feats, int64_t capacity,
                     int64_t* n_out) {
  const int64_t nb = (n + kSubBlock - 1) / kSubBlock;
  uint32_t* bsums = nullptr;
  unsigned long long* dtotal = nullptr;
  int64_t total = 8 * n;
  if (child_mask && n > 0) {
    cudaError_t e = dev_alloc(h, reinterpret_cast<void**>(&bsums), sizeof(uint32_t) * nb + 16);
    if (e != cudaSuccess) return cuda_error(h, e, "subdivide scan buffer");
    dtotal = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(bsums) +
                                                   ((sizeof(uint32_t) * nb + 7) & ~size_t(7)));
    ++h->launches;
    k_subdiv_count<<<static_cast<unsigned>(nb), kSubBlock, 0, h->stream>>>(child_mask, n, bsums);
    ++h->launches;
    k_subdiv_scan<<<1, 1024, 0, h->stream>>>(bsums, nb, dtotal);
    unsigned long long t = 0;
    e = cudaMemcpyAsync(&t, dtotal, sizeof(t), cudaMemcpyDeviceToHost, h->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
    if (e != cudaSuccess) {
      dev_free(h, bsums);
      return cuda_error(h, e, "subdivide count");
    }
    total = static_cast<int64_t>(t);
  }
  *n_out = total;
  sc_status st = SC_OK;
  if (!out_coords || total == 0) {
    // count only
  } else if (total > capacity) {
    st = set_error(h, SC_ERANGE, "subdivide: output capacity is smaller than the number of children");
  } else if (total >= (1ll << 31)) {
    st = set_error(h, SC_ERANGE, "subdivide: more than 2^31 - 1 children");
  } else {
    ++h->launches;
    k_subdiv_write<<<static_cast<unsigned>(nb), kSubBlock, 0, h->stream>>>(
        reinterpret_cast<const int4*>(coords), n, child_mask, bsums, reinterpret_cast<int4*>(out_coords), out_parent);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess && out_feats) {
      const int vecs = row_bytes / 16;
      const int64_t work = total * vecs;
      const int64_t blocks = std::min<int64_t>((work + 255) / 256, static_cast<int64_t>(h->num_sms) * 16);
      ++h->launches;
      k_gather_rows<<<static_cast<unsigned>(std::max<int64_t>(blocks, 1)), 256, 0, h->stream>>>(
          static_cast<const uint4*>(feats), out_parent, total, vecs, static_cast<uint4*>(out_feats));
      e = cudaGetLastError();
    }
    if (e != cudaSuccess) st = cuda_error(h, e, "subdivide launch");
  }
  dev_free(h, bsums);
  return st;
}

}  // namespace sc
