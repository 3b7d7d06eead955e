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

template <typename T>
sc_status launch_rownorm(Handle* h, void* x, int64_t n, int c, float eps, int ln, int silu, const void* res) {
  const int rows_per_block = 8;
  const unsigned grid = static_cast<unsigned>((n + rows_per_block - 1) / rows_per_block);
  ++h->launches;
  k_rownorm<T><<<grid, rows_per_block * 32, 0, h->stream>>>(static_cast<T*>(x), n, c, eps, ln, silu,
                                                            static_cast<const T*>(res));
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
