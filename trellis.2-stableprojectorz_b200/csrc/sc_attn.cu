// Variable-length scaled dot-product attention (the sparse self/cross
// attention of the SLat flow model): for every sequence b of a batch
// concatenated along the token axis (cu_seqlens), every head h and every query
// row i of b,
//   O[i, h] = sum_j softmax_j(scale * Q[i, h] . K[j, h]) V[j, h]
// over the key rows j of sequence b (src/sparse/ops/attention.ts:24-80, which
// runs src/dense/ops/attention.ts per sequence; O = softmax(Q K^T / sqrt(D)) V
// at :2,61).  Q, K, V, O are [tokens, H, 64] rows of bf16 or f16.
//
// One CTA per (128-query tile of one sequence, head), 256 threads:
//   warp 0     TMA producer: the Q tile once, then per 128-key tile the K
//              tile and the V^T tile into a 3-slot ring
//   warp 1     TMEM owner and single-thread MMA issuer:
//              S_j = Q K_j^T  (M 128, N 128, K 64) into TMEM (two buffers),
//              U_j = P_j V_j  (M 128, N 64, K 128) into TMEM (two buffers),
//              S_{j+1} is issued before U_j so the softmax of tile j overlaps
//              the next score MMA
//   warps 4-7  softmax, one query row per thread (TMEM lane): two passes over
//              its S row (row max, then p = 2^(s*scale*log2 e - m) and its
//              sum), P_j as bf16/f16 into shared memory in the MMA's
//              128B-swizzled K-major layout, and the running output
//              O <- O * 2^(m_old - m_new) + U kept in registers (folded one
//              tile late, so U_j's MMA overlaps the softmax of tile j+1)
// Every operand the MMA reads is K-major: V is first transposed per head into
// V^T [H, 64, keys], each sequence starting at a multiple of 8 keys so every
// TMA inner coordinate is 16-byte aligned.  Key columns past the sequence end
// get p = 0.  Every mbarrier wait is bounded (SC_ETIMEOUT).
#include "sc_common.cuh"
#include "sc_internal.h"

#include <cuda.h>
#include <algorithm>
#include <type_traits>
#include <vector>

namespace sc {

bool make_map_3d(CUtensorMap* m, bool bf16, const void* base, const uint64_t dims[3], const uint64_t strides[2],
                 const uint32_t box[3]);  // sc_conv_tc.cu

namespace {

constexpr int kAttnD = 64;          // head dim
constexpr int kAttnTile = 128;      // query rows per CTA and keys per step
constexpr int kAttnStages = 3;      // K / V^T ring
constexpr int kAttnThreads = 256;
constexpr int kTileBytes = kAttnTile * kAttnD * 2;   // 16 KB: Q, K or V^T tile
constexpr int kPBytes = kAttnTile * kAttnTile * 2;   // 32 KB: P tile (two 64-key atoms)
// shared-memory plan (1024-byte aligned pieces)
constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + kTileBytes;                         // stage s: K at +0, V^T at +16 KB
constexpr int kOffP = kOffKV + kAttnStages * 2 * kTileBytes;       // two P buffers
constexpr int kOffBar = kOffP + 2 * kPBytes;
constexpr int kAttnSmem = kOffBar + 256 + 1024;                    // barriers + alignment slack
constexpr uint32_t kTmemCols = 512;  // S: [0,128) [128,256); U: [256,320) [320,384)

// One per (query tile, head) CTA: the tile's sequence bounds.
struct AttnTile {
  int32_t q0, q1;      // query rows [q0, q1)
  int32_t k0, k1;      // key rows [k0, k1)
  int32_t kp;          // column of key k0 in V^T (a multiple of 8)
  int32_t pad;
};

struct AttnParams {
  const AttnTile* tiles;
  void* out;
  int heads;
  float scale_log2;    // scale * log2(e)
  int* err;
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int32_t c0, int32_t c1, int32_t c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}

template <typename T>
__global__ void __launch_bounds__(kAttnThreads, 1)
    k_attn_fwd(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmVt, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 24);
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t q_full = bar0;
  const uint32_t kv_full0 = bar0 + 8, kv_empty0 = bar0 + 8 * (1 + kAttnStages);
  const uint32_t s_full0 = bar0 + 8 * (1 + 2 * kAttnStages), s_empty0 = s_full0 + 16;
  const uint32_t p_full0 = s_empty0 + 16, u_full0 = p_full0 + 16, u_empty0 = u_full0 + 16;
  const uint32_t done_bar = u_empty0 + 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const AttnTile tile = p.tiles[blockIdx.x];
  const int h = blockIdx.y;
  const int nk = (tile.k1 - tile.k0 + kAttnTile - 1) / kAttnTile;  // key tiles (0: empty key sequence)

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kAttnStages; ++s) {
      mbar_init(kv_full0 + 8 * s, 1);
      mbar_init(kv_empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full0 + 8 * b, 1);
      mbar_init(s_empty0 + 8 * b, 128);
      mbar_init(p_full0 + 8 * b, 128);
      mbar_init(u_full0 + 8 * b, 1);
      mbar_init(u_empty0 + 8 * b, 128);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    // ----------------------------------------------------------- producer
    if (lane == 0 && nk > 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmVt);
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_3d(sbase + kOffQ, &tmQ, 0, h, tile.q0, q_full);
      for (int j = 0; j < nk; ++j) {
        const int st = j % kAttnStages, n = j / kAttnStages;
        if (!mbar_wait(kv_empty0 + 8 * st, (n & 1) ^ 1, p.err)) break;
        const uint32_t kb = sbase + kOffKV + st * 2 * kTileBytes;
        mbar_arrive_expect_tx(kv_full0 + 8 * st, 2 * kTileBytes);
        tma_load_3d(kb, &tmK, 0, h, tile.k0 + j * kAttnTile, kv_full0 + 8 * st);
        // V^T: two 64-key atoms of [64 dims][64 keys]
        tma_load_3d(kb + kTileBytes, &tmVt, tile.kp + j * kAttnTile, 0, h, kv_full0 + 8 * st);
        tma_load_3d(kb + kTileBytes + kTileBytes / 2, &tmVt, tile.kp + j * kAttnTile + 64, 0, h, kv_full0 + 8 * st);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0 && nk > 0) {
      const bool bf16 = std::is_same_v<T, __nv_bfloat16>;
      const uint32_t id_s = idesc_f16(128, 128, bf16), id_u = idesc_f16(128, 64, bf16);
      bool ok = mbar_wait(q_full, 0, p.err);
      auto issue_s = [&](int j) -> bool {  // S_j = Q K_j^T
        const int st = j % kAttnStages, b = j & 1;
        if (!mbar_wait(kv_full0 + 8 * st, (j / kAttnStages) & 1, p.err)) return false;
        if (!mbar_wait(s_empty0 + 8 * b, ((j >> 1) & 1) ^ 1, p.err)) return false;
        tc_fence_after();
        const uint32_t kb = sbase + kOffKV + st * 2 * kTileBytes;
#pragma unroll
        for (int k = 0; k < kAttnD / 16; ++k)
          tc_mma_f16(tmem + b * 128, smem_desc(sbase + kOffQ + 32u * k, 1024, 2), smem_desc(kb + 32u * k, 1024, 2),
                     id_s, k > 0 ? 1u : 0u);
        tc_commit(s_full0 + 8 * b);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < nk; ++j) {
        const int st = j % kAttnStages, b = j & 1;
        if (j + 1 < nk && !issue_s(j + 1)) break;
        if (!mbar_wait(p_full0 + 8 * b, (j >> 1) & 1, p.err)) break;
        if (!mbar_wait(u_empty0 + 8 * b, ((j >> 1) & 1) ^ 1, p.err)) break;
        tc_fence_after();
        const uint32_t pb = sbase + kOffP + b * kPBytes;
        const uint32_t vb = sbase + kOffKV + st * 2 * kTileBytes + kTileBytes;
#pragma unroll
        for (int k = 0; k < kAttnTile / 16; ++k) {
          const uint32_t atom = static_cast<uint32_t>(k >> 2), off = 32u * (k & 3);
          tc_mma_f16(tmem + 256 + b * 64, smem_desc(pb + atom * (kPBytes / 2) + off, 1024, 2),
                     smem_desc(vb + atom * (kTileBytes / 2) + off, 1024, 2), id_u, k > 0 ? 1u : 0u);
        }
        tc_commit(u_full0 + 8 * b);
        tc_commit(kv_empty0 + 8 * st);  // K_j and V_j are no longer read
      }
      // every MMA issued must finish before TMEM is released
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, p.err);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const int qrow = tile.q0 + row;
    float o[kAttnD];
#pragma unroll
    for (int d = 0; d < kAttnD; ++d) o[d] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    bool ok = true;
    uint8_t* const pbase = smem + kOffP;
    // folds U_j (written by the MMA for tile j) into o with alpha_j
    auto fold = [&](int j, float alpha) -> bool {
      const int b = j & 1;
      int w = 1;
      if (lane == 0) w = mbar_wait_sleep<256>(u_full0 + 8 * b, (j >> 1) & 1, p.err) ? 1 : 0;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) return false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < kAttnD / 32; ++c) {
        float u[32];
        tmem_ld32(lane_base + 256 + b * 64 + c * 32, u);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[c * 32 + i] = fmaf(o[c * 32 + i], alpha, u[i]);
      }
      tc_fence_before();
      mbar_arrive(u_empty0 + 8 * b);
      return true;
    };
    for (int j = 0; j < nk; ++j) {
      const int b = j & 1;
      const int kbeg = tile.k0 + j * kAttnTile;
      const int valid = min(kAttnTile, tile.k1 - kbeg);  // key columns of this tile in the sequence
      int w = 1;
      if (lane == 0) w = mbar_wait_sleep<256>(s_full0 + 8 * b, (j >> 1) & 1, p.err) ? 1 : 0;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sa = lane_base + b * 128;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kAttnTile / 32; ++c) {
        float s[32];
        tmem_ld32(sa + c * 32, s);
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = (c * 32 + i < valid) ? fmaxf(mx, s[i]) : mx;
      }
      const float m_new = fmaxf(m, mx * p.scale_log2);
      float sum = 0.f;
      uint8_t* const prow = pbase + b * kPBytes + row * 128;
#pragma unroll
      for (int c = 0; c < kAttnTile / 32; ++c) {
        float s[32];
        tmem_ld32(sa + c * 32, s);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float p0 = (c * 32 + i < valid) ? exp2f(fmaf(s[i], p.scale_log2, -m_new)) : 0.f;
          const float p1 = (c * 32 + i + 1 < valid) ? exp2f(fmaf(s[i + 1], p.scale_log2, -m_new)) : 0.f;
          sum += p0 + p1;
          pk[i / 2] = pack2<T>(p0, p1);
        }
        // 32 keys = four 16-byte chunks of the row, in the 128B swizzle of atom c / 2
        uint8_t* const arow = prow + (c >> 1) * (kPBytes / 2);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int chunk = (c & 1) * 4 + q4;
          *reinterpret_cast<uint4*>(arow + ((chunk ^ (row & 7)) << 4)) =
              make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(s_empty0 + 8 * b);   // S_j is read
      fence_proxy_async_smem();        // P_j (generic stores) is visible to the MMA's async reads
      mbar_arrive(p_full0 + 8 * b);
      const float alpha = exp2f(m - m_new);
      l = fmaf(l, alpha, sum);
      m = m_new;
      if (j > 0 && !fold(j - 1, alpha_prev)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
    }
    if (ok && nk > 0) ok = fold(nk - 1, alpha_prev);
    if (qrow < tile.q1) {
      const float inv = (ok && l > 0.f) ? 1.f / l : 0.f;
      T* dst = static_cast<T*>(p.out) + (static_cast<int64_t>(qrow) * p.heads + h) * kAttnD;
#pragma unroll
      for (int c = 0; c < kAttnD / 8; ++c)
        reinterpret_cast<uint4*>(dst)[c] =
            make_uint4(pack2<T>(o[8 * c] * inv, o[8 * c + 1] * inv), pack2<T>(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                       pack2<T>(o[8 * c + 4] * inv, o[8 * c + 5] * inv), pack2<T>(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// V [tokens, H, 64] -> V^T [H, 64, cols]: token t of sequence b goes to
// column kp[b] + (t - k0[b]).  One block per (64-token chunk, head); rows of
// the chunk that belong to different sequences are placed independently.
template <typename T>
__global__ void __launch_bounds__(256) k_attn_vt(const T* __restrict__ v, const int32_t* __restrict__ col_of_token,
                                                 int64_t tokens, int heads, int64_t cols, T* __restrict__ vt) {
  __shared__ T tile[64][kAttnD + 8];
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * 64;
  const int h = blockIdx.y;
  // load 64 tokens x 64 dims (8 threads per token row, 16 bytes each)
  for (int e = threadIdx.x; e < 64 * 8; e += blockDim.x) {
    const int r = e >> 3, c = e & 7;
    const int64_t t = t0 + r;
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (t < tokens) val = __ldg(reinterpret_cast<const uint4*>(v + (t * heads + h) * kAttnD) + c);
    const T* pv = reinterpret_cast<const T*>(&val);
#pragma unroll
    for (int k = 0; k < 8; ++k) tile[r][c * 8 + k] = pv[k];
  }
  __syncthreads();
  // write dim-major: thread (d, r) writes V^T[h][d][col(t0 + r)]
  for (int e = threadIdx.x; e < 64 * kAttnD; e += blockDim.x) {
    const int d = e >> 6, r = e & 63;
    const int64_t t = t0 + r;
    if (t < tokens) vt[(static_cast<int64_t>(h) * kAttnD + d) * cols + __ldg(col_of_token + t)] = tile[r][d];
  }
}

template <typename T>
sc_status launch_attn(Handle* h, const void* q, const void* k, const void* v, void* out, const int32_t* cu_q,
                      const int32_t* cu_kv, int batch, int heads, float scale) {
  const bool bf16 = std::is_same_v<T, __nv_bfloat16>;
  const int64_t nq = cu_q[batch], nkv = cu_kv[batch];
  // host plan: query tiles, padded V^T columns per sequence, column of every key token
  std::vector<AttnTile> tiles;
  std::vector<int32_t> col(static_cast<size_t>(std::max<int64_t>(nkv, 1)));
  int64_t cols = 0;
  for (int b = 0; b < batch; ++b) {
    const int32_t kp = static_cast<int32_t>(cols);
    for (int64_t t = cu_kv[b]; t < cu_kv[b + 1]; ++t) col[t] = static_cast<int32_t>(kp + (t - cu_kv[b]));
    cols += ((cu_kv[b + 1] - cu_kv[b]) + 7) / 8 * 8;
    for (int32_t q0 = cu_q[b]; q0 < cu_q[b + 1]; q0 += kAttnTile)
      tiles.push_back(AttnTile{q0, std::min(q0 + kAttnTile, cu_q[b + 1]), cu_kv[b], cu_kv[b + 1], kp, 0});
  }
  if (tiles.empty()) return SC_OK;
  if (cols >= (1ll << 31)) return set_error(h, SC_EINVAL, "attention: too many key tokens");
  cols = std::max<int64_t>(cols, 8);
  const size_t tile_bytes = sizeof(AttnTile) * tiles.size();
  const size_t col_bytes = sizeof(int32_t) * col.size();
  const size_t vt_bytes = sizeof(T) * static_cast<size_t>(heads) * kAttnD * static_cast<size_t>(cols);
  uint8_t* buf = nullptr;
  const size_t off_col = (tile_bytes + 255) / 256 * 256, off_vt = off_col + (col_bytes + 255) / 256 * 256;
  cudaError_t e = dev_alloc(h, reinterpret_cast<void**>(&buf), off_vt + vt_bytes);
  if (e != cudaSuccess) return cuda_error(h, e, "attention buffers");
  auto fail = [&](cudaError_t err, const char* what) {
    dev_free(h, buf);
    return cuda_error(h, err, what);
  };
  AttnTile* d_tiles = reinterpret_cast<AttnTile*>(buf);
  int32_t* d_col = reinterpret_cast<int32_t*>(buf + off_col);
  T* vt = reinterpret_cast<T*>(buf + off_vt);
  e = cudaMemcpyAsync(d_tiles, tiles.data(), tile_bytes, cudaMemcpyHostToDevice, h->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(d_col, col.data(), col_bytes, cudaMemcpyHostToDevice, h->stream);
  // padding columns between sequences must be finite: they meet p = 0
  if (e == cudaSuccess) e = cudaMemsetAsync(vt, 0, vt_bytes, h->stream);
  if (e != cudaSuccess) return fail(e, "attention plan copy");
  if (nkv > 0) {
    ++h->launches;
    k_attn_vt<T><<<dim3(static_cast<unsigned>((nkv + 63) / 64), heads), 256, 0, h->stream>>>(
        static_cast<const T*>(v), d_col, nkv, heads, cols, vt);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail(e, "attention V transpose launch");
  }
  CUtensorMap tq, tk, tv;
  const uint64_t row = static_cast<uint64_t>(heads) * kAttnD * 2;
  const uint64_t dq[3] = {kAttnD, static_cast<uint64_t>(heads), static_cast<uint64_t>(std::max<int64_t>(nq, 1))};
  const uint64_t dk[3] = {kAttnD, static_cast<uint64_t>(heads), static_cast<uint64_t>(std::max<int64_t>(nkv, 1))};
  const uint64_t sq[2] = {kAttnD * 2, row};
  const uint32_t bq[3] = {kAttnD, 1, kAttnTile};
  const uint64_t dv[3] = {static_cast<uint64_t>(cols), kAttnD, static_cast<uint64_t>(heads)};
  const uint64_t sv[2] = {static_cast<uint64_t>(cols) * 2, static_cast<uint64_t>(cols) * 2 * kAttnD};
  const uint32_t bv[3] = {64, kAttnD, 1};
  if (!make_map_3d(&tq, bf16, q, dq, sq, bq) || !make_map_3d(&tk, bf16, k, dk, sq, bq) ||
      !make_map_3d(&tv, bf16, vt, dv, sv, bv)) {
    dev_free(h, buf);
    return set_error(h, SC_ECUDA, "cuTensorMapEncodeTiled failed (attention)");
  }
  AttnParams ap{};
  ap.tiles = d_tiles;
  ap.out = out;
  ap.heads = heads;
  ap.scale_log2 = scale * 1.4426950408889634f;
  ap.err = h->derr;
  e = cudaFuncSetAttribute(k_attn_fwd<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
  if (e != cudaSuccess) return fail(e, "attention smem attribute");
  ++h->launches;
  k_attn_fwd<T><<<dim3(static_cast<unsigned>(tiles.size()), heads), kAttnThreads, kAttnSmem, h->stream>>>(tq, tk, tv,
                                                                                                         ap);
  e = cudaGetLastError();
  dev_free(h, buf);  // stream-ordered: released after the kernels that use it
  return e == cudaSuccess ? SC_OK : cuda_error(h, e, "attention launch");
}

}  // namespace

sc_status attention_varlen(Handle* h, const void* q, const void* k, const void* v, void* out, const int32_t* cu_q,
                           const int32_t* cu_kv, int batch, int heads, float scale, sc_dtype dtype) {
  if (dtype == SC_BF16) return launch_attn<__nv_bfloat16>(h, q, k, v, out, cu_q, cu_kv, batch, heads, scale);
  return launch_attn<__half>(h, q, k, v, out, cu_q, cu_kv, batch, heads, scale);
}

}  // namespace sc
