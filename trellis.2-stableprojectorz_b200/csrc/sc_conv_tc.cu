// Fused sparse conv on tcgen05 tensor cores (bf16/f16 in, f32 accumulate).
//
// Implicit GEMM over the kernel map: for each 128-row output tile and each
// neighbour offset v present in the tile,
//     D[128, bn] += gather(feats, gidx[t][v])[128, Ci] . W[:, v, :]^T
// with the gather done by TMA tile::gather4 (four rows per instruction, rows
// of -1 are zero-filled by the TMA unit) and W[:, v, kc] by a tiled TMA load,
// both into 128B/64B/32B-swizzled shared memory that tcgen05.mma reads
// directly.  The accumulator lives in TMEM (two buffers, so the epilogue of
// one tile overlaps the main loop of the next).  The epilogue adds bias and
// optionally LayerNorm / SiLU / residual and stores bf16/f16 rows.
//
// Warp roles (192 threads, one persistent CTA per SM):
//   warp 0     TMA producer (all 32 lanes issue one gather4 each per stage)
//   warp 1     TMEM allocator + single-thread MMA issuer
//   warps 2-5  epilogue (warp w reads TMEM lanes 32*(w%4) .. +31)
//
// Reference math: src/sparse/ops/conv3d_wgsl.ts:177-222 (pass 2), weight
// layout (Co,Kd,Kh,Kw,Ci) from src/sparse/ops/conv3d.ts:5,48-49.  No TMA
// multicast is used anywhere.
#include "sc_common.cuh"
#include "sc_internal.h"

#include <cuda.h>
#include <algorithm>
#include <type_traits>

namespace sc {
namespace {

template <int KC> struct SwizzleCfg;
template <> struct SwizzleCfg<64> {
  static constexpr uint32_t kMode = 2, kSbo = 1024;
  static constexpr CUtensorMapSwizzle kTma = CU_TENSOR_MAP_SWIZZLE_128B;
};
template <> struct SwizzleCfg<32> {
  static constexpr uint32_t kMode = 4, kSbo = 512;
  static constexpr CUtensorMapSwizzle kTma = CU_TENSOR_MAP_SWIZZLE_64B;
};
template <> struct SwizzleCfg<16> {
  static constexpr uint32_t kMode = 6, kSbo = 256;
  static constexpr CUtensorMapSwizzle kTma = CU_TENSOR_MAP_SWIZZLE_32B;
};

struct TcParams {
  const int32_t* gidx;
  const int32_t* tile_rows;
  const uint32_t* tile_mask;
  const void* bias;
  const void* residual;
  void* out;
  int64_t num_items;  // tiles * co_blocks
  int co_blocks;
  int K;
  int ci;
  int co;
  int bn;       // output channels per item (MMA N)
  int nchunks;  // ci / KC
  uint32_t epi;
  float eps;
  int* err;
};

constexpr int kTcThreads = 192;

template <int KC, int BNMAX>
struct TcShape {
  static constexpr int kABytes = 128 * KC * 2;
  static constexpr int kBBytes = BNMAX * KC * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStagesFit = (192 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesFit > 12 ? 12 : kStagesFit;
  static constexpr uint32_t kTmemCols =
      (2 * BNMAX <= 32) ? 32 : (2 * BNMAX <= 64) ? 64 : (2 * BNMAX <= 128) ? 128 : (2 * BNMAX <= 256) ? 256 : 512;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarBytes + 1024;
  static_assert(kStageBytes % 1024 == 0, "stage must keep 1024-byte alignment");
  static_assert(2 * kStages + 5 <= 30, "barrier area too small");
};

template <typename T, int W>
__device__ __forceinline__ void load_row(const T* src, float (&x)[W]) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < W / 8; ++q) {
    const uint4 u = __ldg(s + q);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (std::is_same_v<T, __nv_bfloat16>) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
        x[q * 8 + 2 * j] = f.x;
        x[q * 8 + 2 * j + 1] = f.y;
      } else {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
        x[q * 8 + 2 * j] = f.x;
        x[q * 8 + 2 * j + 1] = f.y;
      }
    }
  }
}

template <typename T, int W>
__device__ __forceinline__ void store_row(T* dst, const float (&x)[W]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < W / 8; ++q) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (std::is_same_v<T, __nv_bfloat16>) {
        const __nv_bfloat162 b = __floats2bfloat162_rn(x[q * 8 + 2 * j], x[q * 8 + 2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&b);
      } else {
        const __half2 b = __floats2half2_rn(x[q * 8 + 2 * j], x[q * 8 + 2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&b);
      }
    }
    d[q] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Sum over W accumulator columns of (acc + bias - shift), squared when `sq`.
template <typename T, int W>
__device__ __forceinline__ float chunk_sum(uint32_t tb, int c0, bool live, const T* bias, int col0, float shift,
                                           bool sq) {
  float v[W];
  tmem_ld<W>(tb + c0, v);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < W; ++j) {
    const float d = (live ? v[j] : 0.f) + (bias ? Cvt<T>::to_f(bias[col0 + c0 + j]) : 0.f) - shift;
    s += sq ? d * d : d;
  }
  return s;
}

// Epilogue of W columns of one output row: +bias, LayerNorm, SiLU, +residual, store.
template <typename T, int W>
__device__ __forceinline__ void epi_chunk(uint32_t tb, int c0, bool live, const T* bias, const T* res, T* out,
                                          int r, int co, int col0, float mean, float rstd, uint32_t epi) {
  float v[W];
  tmem_ld<W>(tb + c0, v);
#pragma unroll
  for (int j = 0; j < W; ++j) {
    float x = (live ? v[j] : 0.f) + (bias ? Cvt<T>::to_f(bias[col0 + c0 + j]) : 0.f);
    if (epi & SC_EPI_LAYERNORM) x = (x - mean) * rstd;
    if (epi & SC_EPI_SILU) x = silu_f(x);
    v[j] = x;
  }
  if (r >= 0) {
    const int64_t off = static_cast<int64_t>(r) * co + col0 + c0;
    if (epi & SC_EPI_RESIDUAL) {
      float rr[W];
      load_row<T, W>(res + off, rr);
#pragma unroll
      for (int j = 0; j < W; ++j) v[j] += rr[j];
    }
    store_row<T, W>(out + off, v);
  }
}

template <int KC, int BNMAX, bool BF16>
__global__ void __launch_bounds__(kTcThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const TcParams p) {
  using S = TcShape<KC, BNMAX>;
  using Z = SwizzleCfg<KC>;
  using T = std::conditional_t<BF16, __nv_bfloat16, __half>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kStages * S::kStageBytes);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 30);
  const uint32_t smem_base = smem_u32(smem);
  const uint32_t bar_base = smem_u32(bars);
  const uint32_t full0 = bar_base;
  const uint32_t empty0 = bar_base + 8u * S::kStages;
  const uint32_t tfull0 = bar_base + 16u * S::kStages;
  const uint32_t tempty0 = tfull0 + 16u;
  const uint32_t done_bar = tfull0 + 32u;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
    }
    mbar_init(tfull0, 1);
    mbar_init(tfull0 + 8u, 1);
    mbar_init(tempty0, 128);
    mbar_init(tempty0 + 8u, 128);
    mbar_init(done_bar, 1);
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int bn = p.bn;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint32_t stage_tx = static_cast<uint32_t>(S::kABytes + bn * KC * 2);
    int stage = 0;
    uint32_t phase = 0;
    uint32_t used = 0, used_par = 0;  // stages ever filled and the parity of their last fill
    bool ok = true;
    for (int64_t item = blockIdx.x; ok && item < p.num_items; item += gridDim.x) {
      const int64_t t = item / p.co_blocks;
      const int cb = static_cast<int>(item - t * p.co_blocks);
      uint32_t mask = __ldg(p.tile_mask + t);
      while (ok && mask) {
        const int v = __ffs(mask) - 1;
        mask &= mask - 1;
        const int4 idx = __ldg(reinterpret_cast<const int4*>(p.gidx + (t * p.K + v) * 128) + lane);
        for (int kc = 0; kc < p.nchunks; ++kc) {
          int w = 1;
          if (lane == 0) w = mbar_wait(empty0 + 8u * stage, phase ^ 1u, p.err) ? 1 : 0;
          w = __shfl_sync(0xffffffffu, w, 0);
          if (!w) {
            ok = false;
            break;
          }
          if (lane == 0) mbar_arrive_expect_tx(full0 + 8u * stage, stage_tx);
          __syncwarp();
          const uint32_t sbase = smem_base + static_cast<uint32_t>(stage * S::kStageBytes);
          tma_gather4(sbase + static_cast<uint32_t>(lane * 4 * KC * 2), &tmA, kc * KC, idx.x, idx.y, idx.z, idx.w,
                      full0 + 8u * stage);
          if (lane == 0) tma_load_2d(sbase + S::kABytes, &tmB, v * p.ci + kc * KC, cb * bn, full0 + 8u * stage);
          used |= 1u << stage;
          used_par = (used_par & ~(1u << stage)) | (phase << stage);
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    if (!ok && lane == 0) {
      // Error exit: let copies already issued into our shared memory land.
      for (int s = 0; s < S::kStages; ++s)
        if (used & (1u << s)) mbar_wait(full0 + 8u * s, (used_par >> s) & 1u, nullptr);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, bn, BF16);
      int stage = 0;
      uint32_t phase = 0, it = 0;
      bool ok = true;
      for (int64_t item = blockIdx.x; ok && item < p.num_items; item += gridDim.x, ++it) {
        const int64_t t = item / p.co_blocks;
        const uint32_t acc = it & 1u, aph = (it >> 1) & 1u;
        if (!mbar_wait(tempty0 + 8u * acc, aph ^ 1u, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * static_cast<uint32_t>(BNMAX);
        const int nsteps = __popc(__ldg(p.tile_mask + t)) * p.nchunks;
        for (int s = 0; s < nsteps; ++s) {
          if (!mbar_wait(full0 + 8u * stage, phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_base + static_cast<uint32_t>(stage * S::kStageBytes);
          const uint32_t b0 = a0 + S::kABytes;
#pragma unroll
          for (int k = 0; k < KC / 16; ++k) {
            tc_mma_f16(d_tmem, smem_desc(a0 + 32u * k, Z::kSbo, Z::kMode), smem_desc(b0 + 32u * k, Z::kSbo, Z::kMode),
                       idesc, (s > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(empty0 + 8u * stage);
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(tfull0 + 8u * acc);
      }
      // All MMAs issued by this thread must finish before TMEM is released.
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, p.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const T* bias = static_cast<const T*>(p.bias);
    const T* res = static_cast<const T*>(p.residual);
    T* out = static_cast<T*>(p.out);
    uint32_t it = 0;
    for (int64_t item = blockIdx.x; item < p.num_items; item += gridDim.x, ++it) {
      const int64_t t = item / p.co_blocks;
      const int cb = static_cast<int>(item - t * p.co_blocks);
      const uint32_t acc = it & 1u, aph = (it >> 1) & 1u;
      int w = 1;
      if (lane == 0) w = mbar_wait(tfull0 + 8u * acc, aph, p.err) ? 1 : 0;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) break;
      tc_fence_after();
      const int r = __ldg(p.tile_rows + t * 128 + row);
      const bool live = __ldg(p.tile_mask + t) != 0u;
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * static_cast<uint32_t>(BNMAX);
      const int col0 = cb * bn;
      const int bn32 = bn & ~31;  // columns handled 32 at a time; a 16-wide tail follows when bn % 32 == 16
      float mean = 0.f, rstd = 1.f;
      if (p.epi & SC_EPI_LAYERNORM) {
        float s1 = 0.f;
        for (int c0 = 0; c0 < bn32; c0 += 32) s1 += chunk_sum<T, 32>(tb, c0, live, bias, col0, 0.f, false);
        if (bn32 < bn) s1 += chunk_sum<T, 16>(tb, bn32, live, bias, col0, 0.f, false);
        mean = s1 / static_cast<float>(bn);
        float s2 = 0.f;
        for (int c0 = 0; c0 < bn32; c0 += 32) s2 += chunk_sum<T, 32>(tb, c0, live, bias, col0, mean, true);
        if (bn32 < bn) s2 += chunk_sum<T, 16>(tb, bn32, live, bias, col0, mean, true);
        rstd = rsqrtf(s2 / static_cast<float>(bn) + p.eps);
      }
      for (int c0 = 0; c0 < bn32; c0 += 32) epi_chunk<T, 32>(tb, c0, live, bias, res, out, r, p.co, col0, mean, rstd, p.epi);
      if (bn32 < bn) epi_chunk<T, 16>(tb, bn32, live, bias, res, out, r, p.co, col0, mean, rstd, p.epi);
      tc_fence_before();
      mbar_arrive(tempty0 + 8u * acc);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

// --------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn lookup_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<EncodeTiledFn>(fn);
}

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = lookup_encode();
  return fn;
}

bool make_map_2d(CUtensorMap* m, bool bf16, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
             const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int KC, int BNMAX, bool BF16>
sc_status launch_tc(Handle* h, const KMap* km, const void* feats, const void* weight, TcParams p) {
  using S = TcShape<KC, BNMAX>;
  using Z = SwizzleCfg<KC>;
  CUtensorMap ta, tb;
  if (!make_map_2d(&ta, BF16, feats, p.ci, km->n_in, static_cast<uint64_t>(p.ci) * 2, KC, 1, Z::kTma) ||
      !make_map_2d(&tb, BF16, weight, static_cast<uint64_t>(km->K) * p.ci, p.co,
                   static_cast<uint64_t>(km->K) * p.ci * 2, KC, p.bn, Z::kTma))
    return set_error(h, SC_ECUDA, "cuTensorMapEncodeTiled failed");
  auto kern = conv_tc_kernel<KC, BNMAX, BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes);
  if (e != cudaSuccess) return cuda_error(h, e, "conv smem attribute");
  const int64_t grid = std::min<int64_t>(p.num_items, h->num_sms);
  kern<<<static_cast<unsigned>(grid), kTcThreads, S::kSmemBytes, h->stream>>>(ta, tb, p);
  e = cudaGetLastError();
  return e == cudaSuccess ? SC_OK : cuda_error(h, e, "conv launch");
}

template <int KC, bool BF16>
sc_status dispatch_bn(Handle* h, const KMap* km, const void* feats, const void* weight, const TcParams& p) {
  if (p.bn <= 64) return launch_tc<KC, 64, BF16>(h, km, feats, weight, p);
  if (p.bn <= 128) return launch_tc<KC, 128, BF16>(h, km, feats, weight, p);
  return launch_tc<KC, 256, BF16>(h, km, feats, weight, p);
}

template <bool BF16>
sc_status dispatch_kc(Handle* h, const KMap* km, const void* feats, const void* weight, TcParams p) {
  if (p.ci % 64 == 0) {
    p.nchunks = p.ci / 64;
    return dispatch_bn<64, BF16>(h, km, feats, weight, p);
  }
  if (p.ci % 32 == 0) {
    p.nchunks = p.ci / 32;
    return dispatch_bn<32, BF16>(h, km, feats, weight, p);
  }
  p.nchunks = p.ci / 16;
  return dispatch_bn<16, BF16>(h, km, feats, weight, p);
}

inline bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

__global__ void k_check_gidx(const int32_t* gidx, int64_t total, int64_t n_in, int* err) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < total) {
    const int32_t r = gidx[i];
    if (r < -1 || r >= n_in) record_error(err, SC_EINVAL);
  }
}

}  // namespace

// Debug mode: verifies every gather index of the map lies in [-1, n_in).
sc_status check_gather_bounds(Handle* h, const KMap* km) {
  const int64_t total = km->num_tiles * km->K * kTileRows;
  if (total == 0) return SC_OK;
  int* derr = nullptr;
  cudaError_t e = dev_alloc(h, reinterpret_cast<void**>(&derr), 16);
  if (e != cudaSuccess) return cuda_error(h, e, "bounds check alloc");
  int herr = 0;
  e = cudaMemsetAsync(derr, 0, 16, h->stream);
  if (e == cudaSuccess) {
    k_check_gidx<<<static_cast<unsigned>((total + 255) / 256), 256, 0, h->stream>>>(km->gidx, total, km->n_in, derr);
    e = cudaMemcpyAsync(&herr, derr, 4, cudaMemcpyDeviceToHost, h->stream);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  dev_free(h, derr);
  if (e != cudaSuccess) return cuda_error(h, e, "bounds check");
  if (herr) return set_error(h, SC_EINVAL, "gather index out of range");
  return SC_OK;
}

sc_status conv_tc(Handle* h, const KMap* km, const void* feats, const void* weight, const void* bias,
                  const void* residual, void* out, int ci, int co, sc_dtype dtype, uint32_t epi, float eps) {
  if (ci % 16 != 0 || co % 16 != 0)
    return set_error(h, SC_EUNSUPPORTED, "bf16/f16 conv needs Ci and Co multiples of 16");
  if (km->n_in <= 0) return set_error(h, SC_EINVAL, "map has no input rows");
  if (!al16(feats) || !al16(weight) || !al16(out) || (residual && !al16(residual)) ||
      (bias && (reinterpret_cast<uintptr_t>(bias) & 1u)))
    return set_error(h, SC_EINVAL, "feats/weight/out/residual must be 16-byte aligned");
  int bn = co;
  if (co > 256) {
    bn = 0;
    for (int b = 256; b >= 16; b -= 16)
      if (co % b == 0) {
        bn = b;
        break;
      }
  }
  if ((epi & SC_EPI_LAYERNORM) && bn != co) return set_error(h, SC_EUNSUPPORTED, "fused LayerNorm needs Co <= 256");
  if (h->debug_bounds) {
    const sc_status st = check_gather_bounds(h, km);
    if (st != SC_OK) return st;
  }
  TcParams p{};
  p.gidx = km->gidx;
  p.tile_rows = km->tile_rows;
  p.tile_mask = km->tile_mask;
  p.bias = bias;
  p.residual = residual;
  p.out = out;
  p.co_blocks = co / bn;
  p.num_items = km->num_tiles * p.co_blocks;
  p.K = km->K;
  p.ci = ci;
  p.co = co;
  p.bn = bn;
  p.epi = epi;
  p.eps = eps;
  p.err = h->derr;
  if (p.num_items == 0) return SC_OK;
  return dtype == SC_BF16 ? dispatch_kc<true>(h, km, feats, weight, p)
                          : dispatch_kc<false>(h, km, feats, weight, p);
}

}  // namespace sc
