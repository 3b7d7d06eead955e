// f32 sparse conv (FFMA) and row LayerNorm / SiLU.
//
// The f32 path keeps the reference's f32 arithmetic (conv3d_wgsl.ts:177-222
// with T = f32) so its result matches a float64 restatement to ~1e-7
// relative L2; tensor-core tf32 would not.  It reuses the tile layout of the
// kernel map: per 128-row tile and offset, the gathered rows and the weight
// slice are staged in shared memory in 32-channel chunks and contracted with
// an 8x4 register tile per thread.
#include "sc_common.cuh"
#include "sc_internal.h"

#include <type_traits>

namespace sc {
namespace {

constexpr int kSimtCo = 64;     // output channels per block
constexpr int kSimtCi = 32;     // input channels per shared-memory chunk

__global__ void __launch_bounds__(256) k_conv_simt_f32(const int32_t* __restrict__ gidx,
                                                        const int32_t* __restrict__ tile_rows,
                                                        const uint32_t* __restrict__ tile_mask, int K, int co_blocks,
                                                        const float* __restrict__ feats,
                                                        const float* __restrict__ weight,
                                                        const float* __restrict__ bias,
                                                        const float* __restrict__ residual,
                                                        float* __restrict__ out, int ci, int co, uint32_t epi) {
  __shared__ float sA[kSimtCi][kTileRows + 4];
  __shared__ float sW[kSimtCi][kSimtCo + 4];
  __shared__ int sIdx[kTileRows];
  const int64_t t = blockIdx.x / co_blocks;
  const int cb = static_cast<int>(blockIdx.x - t * co_blocks);
  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;  // rows ty*8..+7, cols tx*4..+3
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  uint32_t mask = tile_mask[t];
  while (mask) {
    const int v = __ffs(mask) - 1;
    mask &= mask - 1;
    __syncthreads();
    if (tid < kTileRows) sIdx[tid] = gidx[(t * K + v) * kTileRows + tid];
    __syncthreads();
    for (int c0 = 0; c0 < ci; c0 += kSimtCi) {
      {
        const int r = tid >> 1, cbase = (tid & 1) * 16;
        const int idx = sIdx[r];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int c = cbase + j;
          sA[c][r] = (idx >= 0 && c0 + c < ci) ? __ldg(feats + static_cast<int64_t>(idx) * ci + c0 + c) : 0.f;
        }
      }
      {
        const int o = tid >> 2, cbase = (tid & 3) * 8;
        const int oc = cb * kSimtCo + o;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int c = cbase + j;
          sW[c][o] = (oc < co && c0 + c < ci)
                         ? __ldg(weight + (static_cast<int64_t>(oc) * K + v) * ci + c0 + c)
                         : 0.f;
        }
      }
      __syncthreads();
#pragma unroll 8
      for (int c = 0; c < kSimtCi; ++c) {
        float a[8], b[4];
#pragma unroll
        for (int i = 0; i < 8; ++i) a[i] = sA[c][ty * 8 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = sW[c][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = tile_rows[t * kTileRows + ty * 8 + i];
    if (r < 0) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int oc = cb * kSimtCo + tx * 4 + j;
      if (oc >= co) continue;
      float x = acc[i][j] + (bias ? bias[oc] : 0.f);
      if (epi & SC_EPI_SILU) x = silu_f(x);
      if (epi & SC_EPI_RESIDUAL) x += residual[static_cast<int64_t>(r) * co + oc];
      out[static_cast<int64_t>(r) * co + oc] = x;
    }
  }
}

// One warp per row: x <- [LayerNorm(x)] -> [SiLU] -> [+ residual].
template <typename T>
__global__ void k_rownorm(T* __restrict__ x, int64_t n, int c, float eps, int do_ln, int do_silu,
                          const T* __restrict__ residual) {
  const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  T* xr = x + row * c;
  float mean = 0.f, rstd = 1.f;
  if (do_ln) {
    float s = 0.f;
    for (int j = lane; j < c; j += 32) s += Cvt<T>::to_f(xr[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    mean = s / static_cast<float>(c);
    float s2 = 0.f;
    for (int j = lane; j < c; j += 32) {
      const float d = Cvt<T>::to_f(xr[j]) - mean;
      s2 += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    rstd = rsqrtf(s2 / static_cast<float>(c) + eps);
  }
  for (int j = lane; j < c; j += 32) {
    float y = Cvt<T>::to_f(xr[j]);
    if (do_ln) y = (y - mean) * rstd;
    if (do_silu) y = silu_f(y);
    if (residual) y += Cvt<T>::to_f(residual[row * c + j]);
    xr[j] = Cvt<T>::from_f(y);
  }
}

// Vectorised rows: L lanes share a row (32 / L rows per warp), each lane
// holds VPL 16-byte vectors of it in registers, so the row is read once and
// written once.  Mean and variance are two passes over the registers (the
// same two-pass statistics as k_rownorm), reduced with xor shuffles inside
// the L-lane group.  Needs c a multiple of the vector width and 16-byte
// aligned rows.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& u, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y); f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  } else {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const T* h = reinterpret_cast<const T*>(&w[j]);
      f[2 * j] = Cvt<T>::to_f(h[0]);
      f[2 * j + 1] = Cvt<T>::to_f(h[1]);
    }
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack16(const float* f) {
  if constexpr (sizeof(T) == 4) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  } else {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (std::is_same_v<T, __nv_bfloat16>) {
        const __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&b);
      } else {
        const __half2 b = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&b);
      }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <typename T, int L, int VPL>
__global__ void __launch_bounds__(256) k_rownorm_vec(T* __restrict__ x, int64_t n, int c, float eps, int do_ln,
                                                     int do_silu, const T* __restrict__ residual) {
  constexpr int EPV = 16 / static_cast<int>(sizeof(T));
  const int lane = threadIdx.x & 31;
  const int li = lane % L;
  const int64_t row = (blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5)) * (32 / L) + lane / L;
  const bool live = row < n;
  const int nvec = c / EPV;
  float v[VPL][EPV];
  uint4* xr = reinterpret_cast<uint4*>(x + (live ? row : 0) * c);
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int j = li + k * L;
    if (live && j < nvec) {
      unpack16<T>(xr[j], v[k]);
    } else {
#pragma unroll
      for (int e = 0; e < EPV; ++e) v[k][e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < EPV; ++e) s += v[k][e];
  }
  float mean = 0.f, rstd = 1.f;
  if (do_ln) {
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    mean = s / static_cast<float>(c);
    float s2 = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      if (li + k * L < nvec) {
#pragma unroll
        for (int e = 0; e < EPV; ++e) {
          const float d = v[k][e] - mean;
          s2 += d * d;
        }
      }
    }
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    rstd = rsqrtf(s2 / static_cast<float>(c) + eps);
  }
  if (!live) return;
  const uint4* rr = residual ? reinterpret_cast<const uint4*>(residual + row * c) : nullptr;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int j = li + k * L;
    if (j >= nvec) continue;
    float y[EPV], r[EPV];
    if (rr) unpack16<T>(rr[j], r);
#pragma unroll
    for (int e = 0; e < EPV; ++e) {
      float t = v[k][e];
      if (do_ln) t = (t - mean) * rstd;
      if (do_silu) t = silu_f(t);
      if (rr) t += r[e];
      y[e] = t;
    }
    xr[j] = pack16<T>(y);
  }
}

template <typename T, int L, int VPL>
void launch_rownorm_vec(Handle* h, T* x, int64_t n, int c, float eps, int ln, int silu, const T* res) {
  const int64_t rows_per_block = 8 * (32 / L);
  const unsigned grid = static_cast<unsigned>((n + rows_per_block - 1) / rows_per_block);
  k_rownorm_vec<T, L, VPL><<<grid, 256, 0, h->stream>>>(x, n, c, eps, ln, silu, res);
}

template <typename T>
sc_status launch_rownorm(Handle* h, void* x, int64_t n, int c, float eps, int ln, int silu, const void* res) {
  constexpr int EPV = 16 / static_cast<int>(sizeof(T));
  const int nvec = c / EPV;
  const bool vec = c % EPV == 0 && nvec >= 4 && nvec <= 32 * 16 &&
                   reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(res) % 16 == 0;
  T* xt = static_cast<T*>(x);
  const T* rt = static_cast<const T*>(res);
  ++h->launches;
  if (vec) {
    const int L = nvec >= 32 ? 32 : nvec >= 16 ? 16 : nvec >= 8 ? 8 : 4;
    const int vpl = (nvec + L - 1) / L;  // <= 2 when L < 32
    if (L == 4) {
      if (vpl == 1) launch_rownorm_vec<T, 4, 1>(h, xt, n, c, eps, ln, silu, rt);
      else launch_rownorm_vec<T, 4, 2>(h, xt, n, c, eps, ln, silu, rt);
    } else if (L == 8) {
      if (vpl == 1) launch_rownorm_vec<T, 8, 1>(h, xt, n, c, eps, ln, silu, rt);
      else launch_rownorm_vec<T, 8, 2>(h, xt, n, c, eps, ln, silu, rt);
    } else if (L == 16) {
      if (vpl == 1) launch_rownorm_vec<T, 16, 1>(h, xt, n, c, eps, ln, silu, rt);
      else launch_rownorm_vec<T, 16, 2>(h, xt, n, c, eps, ln, silu, rt);
    } else if (vpl == 1) {
      launch_rownorm_vec<T, 32, 1>(h, xt, n, c, eps, ln, silu, rt);
    } else if (vpl == 2) {
      launch_rownorm_vec<T, 32, 2>(h, xt, n, c, eps, ln, silu, rt);
    } else if (vpl <= 4) {
      launch_rownorm_vec<T, 32, 4>(h, xt, n, c, eps, ln, silu, rt);
    } else if (vpl <= 8) {
      launch_rownorm_vec<T, 32, 8>(h, xt, n, c, eps, ln, silu, rt);
    } else {
      launch_rownorm_vec<T, 32, 16>(h, xt, n, c, eps, ln, silu, rt);
    }
  } else {
    const int rows_per_block = 8;
    const unsigned grid = static_cast<unsigned>((n + rows_per_block - 1) / rows_per_block);
    k_rownorm<T><<<grid, rows_per_block * 32, 0, h->stream>>>(xt, n, c, eps, ln, silu, rt);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SC_OK : cuda_error(h, e, "rownorm launch");
}

sc_status rownorm(Handle* h, void* x, int64_t n, int c, sc_dtype dtype, float eps, int ln, int silu,
                  const void* res) {
  switch (dtype) {
    case SC_F32: return launch_rownorm<float>(h, x, n, c, eps, ln, silu, res);
    case SC_BF16: return launch_rownorm<__nv_bfloat16>(h, x, n, c, eps, ln, silu, res);
    case SC_F16: return launch_rownorm<__half>(h, x, n, c, eps, ln, silu, res);
  }
  return set_error(h, SC_EINVAL, "unknown dtype");
}

}  // namespace

sc_status conv_simt_f32(Handle* h, const KMap* km, const float* feats, const float* weight, const float* bias,
                        const float* residual, float* out, int ci, int co, uint32_t epi, float eps) {
  if (h->debug_bounds) {
    const sc_status st = check_gather_bounds(h, km);
    if (st != SC_OK) return st;
  }
  const int co_blocks = (co + kSimtCo - 1) / kSimtCo;
  const int64_t blocks = km->num_tiles * co_blocks;
  if (blocks == 0) return SC_OK;
  if (blocks > 0x7fffffffll) return set_error(h, SC_EINVAL, "too many tiles");
  // With LayerNorm the conv writes bias-added rows and the row kernel applies
  // LN -> SiLU -> residual; otherwise the epilogue is fused.
  const bool ln = (epi & SC_EPI_LAYERNORM) != 0;
  ++h->launches;
  k_conv_simt_f32<<<static_cast<unsigned>(blocks), 256, 0, h->stream>>>(
      km->gidx, km->tile_rows, km->tile_mask, km->K, co_blocks, feats, weight, bias, residual, out, ci, co,
      ln ? 0u : epi);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(h, e, "f32 conv launch");
  if (ln)
    return rownorm(h, out, km->n_out, co, SC_F32, eps, 1, (epi & SC_EPI_SILU) ? 1 : 0,
                   (epi & SC_EPI_RESIDUAL) ? residual : nullptr);
  return SC_OK;
}

sc_status layernorm_silu(Handle* h, void* x, int64_t n, int c, sc_dtype dtype, int silu, float eps) {
  return rownorm(h, x, n, c, dtype, eps, 1, silu, nullptr);
}

}  // namespace sc
