// Variable-length scaled dot-product attention (the sparse self/cross
// attention of the SLat flow model): for every sequence b of a batch
// concatenated along the token axis (cu_seqlens), every head h and every query
// row i of b,
//   O[i, h] = sum_j softmax_j(scale * Q[i, h] . K[j, h]) V[j, h]
// over the key rows j of sequence b (src/sparse/ops/attention.ts:24-80, which
// runs src/dense/ops/attention.ts per sequence; O = softmax(Q K^T / sqrt(D)) V
// at :2,61).  Q, K, V, O are [tokens, H, 64] rows of bf16 or f16.
//
// One CTA per (256 query rows of one sequence, head), 384 threads:
//   warp 0     TMA producer: the two 128-row Q tiles once, then per 128-key
//              tile the K tile and the V tile into a 4-slot ring.  Q, K and
//              V are read where they lie, [tokens, H, 64], by 3-D boxes of
//              128 rows of one head
//   warp 1     TMEM owner and single-thread MMA issuer over the steps
//              i = j * groups + g (key tile j, query group g): S of step i
//              = Q_g K_j^T goes into one of three 128-column S buffers shared
//              by the groups (buffer i % 3); when group g's softmax has
//              written P over the first 64 columns of that buffer, O_g +=
//              P V_j reads P as its A operand from tensor memory and V from
//              shared memory as an MN-major operand, and once that product is
//              done, S of step i + 3 goes into the freed buffer.  So a group
//              usually finds its next S computed while it still works on the
//              current tile, and the tensor core alternates between the
//              groups (S: M 128, N 128, K 64; PV: M 128, N 64, K 128; f32
//              accumulators in tensor memory)
//   warp 2     the last key tile of a sequence also holds rows of the next
//              one: their weights are 0, and this warp zeroes their V rows
//              in shared memory (0 * NaN would be NaN)
//   warps 4-7, 8-11  softmax groups 0 and 1, one query row per thread (TMEM
//              lane): two passes over its S row (row max, then
//              p = 2^(s*scale*log2 e - m) and its sum), P as packed bf16/f16
//              pairs over the S columns already read.  The output O
//              accumulates in tensor memory across key tiles; its row max m
//              moves only when a tile's max exceeds it by more than 2^8
//              (conditional rescaling, the running-max trick of
//              FlashAttention-4), and only then is the row of O rescaled
//              in tensor memory.
// Every mbarrier wait is bounded (SC_ETIMEOUT).
//
// Measured on B200, 32k tokens x 16 heads in one sequence: 691-708 TFLOP/s;
// the 10,000 + 6,384-token call 0.94-0.95 ms (0.954 with all 128 softmax
// threads arriving on the P barrier instead of one per warp).  Earlier
// layouts, at 32k:
//   * V transposed per head into a K-major V^T by a separate pass first:
//     711, the 16k-token call 0.99 ms (the pass took 27 us and a zeroed
//     buffer the size of V);
//   * one S buffer per group, the group's next S issued right after its P
//     was written (before its P V) 625, after its P V 563;
//   * P staged in shared memory in the 128B swizzle (eight 16-byte stores
//     per 64 keys and a proxy fence per tile instead of one tcgen05.st) 540;
//     before the packed f32x2 arithmetic of the weight loop 532.
// Measured and dropped:
//   * one in eight / four of the weights from a cubic 2^f polynomial on the
//     FMA pipe instead of ex2 (FlashAttention-4's offload; packed f32x2,
//     fitted to 7.5e-5 relative error): 637 / 564 against 711 with the S
//     ring (507 / 492 against 540 with the first layout): the softmax is
//     bound by its instruction stream, not by the ex2 unit;
//   * 64-key tiles with S double-buffered per group: 428 (the fixed per-tile
//     costs double, and an N = 64 product reads more shared memory per FLOP
//     than N = 128);
//   * keys 64..127 of S kept in registers from the row-max pass to the weight
//     pass (one TMEM read fewer per tile): 698-720, no change;
//   * two threads per query row (eight softmax warps per group, each on 64
//     of a tile's 128 keys, half-row maxima exchanged through shared memory
//     under a named barrier per tile): 596 against 691, the 16k-token call
//     1.087 against 0.956 ms.
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
constexpr int kAttnTile = 128;      // query rows per softmax group and keys per step
constexpr int kAttnStages = 4;      // K / V ring
constexpr int kAttnThreads = 384;   // 12 warps: producer, MMA, V tail, idle, 2 softmax groups of 4
constexpr int kTileBytes = kAttnTile * kAttnD * 2;   // 16 KB: Q, K or V tile
// shared-memory plan (1024-byte aligned pieces)
constexpr int kOffQ = 0;                                           // Q of group 0, group 1 at +16 KB
constexpr int kOffKV = kOffQ + 2 * kTileBytes;                     // stage s: K at +0, V at +16 KB
constexpr int kOffBar = kOffKV + kAttnStages * 2 * kTileBytes;
constexpr int kAttnSmem = kOffBar + 256 + 1024;                    // barriers + alignment slack
// Tensor memory: a ring of three 128-column S buffers at [128b, 128b+128)
// shared by the two groups (S of step i = j * groups + g in buffer i % 3; the
// softmax overwrites the first 64 columns with P, two 16-bit weights per
// 32-bit column), and O of group g at [384+64g, 448+64g).
constexpr int kSBufs = 3;
constexpr uint32_t kTmemCols = 512;
// Conditional rescaling: the running row max used for the exponentials moves
// only when a tile's max exceeds it by more than 2^8, so most tiles leave the
// output accumulator in tensor memory untouched; weights stay below 2^8.
constexpr float kRescaleLog2 = 8.f;

// One per CTA: up to 256 query rows of one sequence (group g takes rows
// q0 + 128g ..) and the sequence's key rows.
struct AttnTile {
  int32_t q0, q1;      // query rows [q0, min(q0 + 256, q1))
  int32_t k0, k1;      // key rows [k0, k1)
  int32_t pad0, pad1;
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

// 2^x with the hardware approximation (2 ulp), subnormal results flushed to
// zero: softmax weights that small contribute nothing at bf16/f16 precision.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed two-wide f32 arithmetic of sm_100 (one instruction per pair).
__device__ __forceinline__ unsigned long long f2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_split(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long fma_f2(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long add_f2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// max(a, b, c) in one instruction (three-input max.f32 of sm_100).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
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

// Each lane reads 64 consecutive f32 columns of its own TMEM lane (one
// instruction, one wait).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// One softmax group (four warps, one query row per thread = TMEM lane):
// for every key tile, the row max of S (two 64-column reads), conditional
// rescaling of the output accumulator O in tensor memory, the weights
// p = 2^(s * scale * log2 e - m) as bf16/f16 pairs written over the first
// 64 columns of the same S buffer (lane = query row, the A operand layout of
// the second product), and the running sum; at the end O / sum to global
// memory.  s_full0 / p_full0: the three S buffers' barriers; o_done: this
// group's "P V done" barrier.
template <typename T>
__device__ __forceinline__ void softmax_group(const AttnParams& p, const AttnTile& tile, int h, int nk, int g,
                                              int ng, int quad, int lane, uint32_t tmem, uint32_t s_full0,
                                              uint32_t p_full0, uint32_t o_done) {
  const int row = quad * 32 + lane;
  const int qrow = tile.q0 + g * kAttnTile + row;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
  const uint32_t oa = lane_base + 384u + g * 64;
  float m = -INFINITY, l = 0.f;
  bool ok = true;
  auto wait_warp = [&](uint32_t bar, uint32_t parity) -> bool {
    int w = 1;
    if (lane == 0) w = mbar_wait(bar, parity, p.err) ? 1 : 0;
    return __shfl_sync(0xffffffffu, w, 0) != 0;
  };
  for (int j = 0; j < nk; ++j) {
    const int valid = min(kAttnTile, tile.k1 - (tile.k0 + j * kAttnTile));  // key columns in the sequence
    const bool full = valid == kAttnTile;                                    // warp-uniform
    const int step = j * ng + g;
    const uint32_t b = static_cast<uint32_t>(step % kSBufs), use = static_cast<uint32_t>(step / kSBufs);
    const uint32_t sa = lane_base + 128u * b;
    if (!wait_warp(s_full0 + 8u * b, use & 1u)) {
      ok = false;
      break;
    }
    tc_fence_after();
    // eight independent max chains (a single chain is 128 dependent steps)
    float mxv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) mxv[k] = -INFINITY;
#pragma unroll
    for (int c = 0; c < kAttnTile / 64; ++c) {
      float s[64];
      tmem_ld64(sa + c * 64, s);
      if (full) {
#pragma unroll
        for (int i = 0; i < 64; i += 2) mxv[(i >> 1) & 7] = max3(mxv[(i >> 1) & 7], s[i], s[i + 1]);
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) mxv[i & 7] = (c * 64 + i < valid) ? fmaxf(mxv[i & 7], s[i]) : mxv[i & 7];
      }
    }
    const float mx = fmaxf(fmaxf(fmaxf(mxv[0], mxv[1]), fmaxf(mxv[2], mxv[3])),
                           fmaxf(fmaxf(mxv[4], mxv[5]), fmaxf(mxv[6], mxv[7])));
    const float m_tile = mx * p.scale_log2;
    const bool move = m_tile > m + kRescaleLog2;  // always true on the first tile (m = -inf)
    const float m_new = move ? m_tile : m;
    const float alpha = move ? ex2_ftz(m - m_new) : 1.f;
    // A rescale waits for O_g to hold the sum through tile j-1.  The S
    // buffer itself was free when S_g(j) was issued into it (the product that
    // last read its P was done), and P_g(j) goes there.
    if (j > 0 && __any_sync(0xffffffffu, move)) {
      if (!wait_warp(o_done, (j - 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float o[64];
      tmem_ld64(oa, o);
      uint32_t w[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(o[half * 32 + i] * alpha);
        tmem_st32(oa + half * 32, w);
      }
      tmem_wait_st();
    }
    unsigned long long sumv[4];  // pairs of partial sums
#pragma unroll
    for (int k = 0; k < 4; ++k) sumv[k] = 0ull;
    const unsigned long long sc2 = f2(p.scale_log2, p.scale_log2), neg_m2 = f2(-m_new, -m_new);
#pragma unroll
    for (int c = 0; c < kAttnTile / 64; ++c) {
      float s[64];
      tmem_ld64(sa + c * 64, s);
      if (!full) {
#pragma unroll
        for (int i = 0; i < 64; ++i) s[i] = (c * 64 + i < valid) ? s[i] : -INFINITY;  // 2^-inf = 0
      }
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        float x0, x1;
        f2_split(fma_f2(f2(s[i], s[i + 1]), sc2, neg_m2), x0, x1);
        const float p0 = ex2_ftz(x0), p1 = ex2_ftz(x1);
        const unsigned long long pp = f2(p0, p1);
        sumv[(i >> 1) & 3] = add_f2(sumv[(i >> 1) & 3], pp);
        pk[i / 2] = pack2<T>(p0, p1);
      }
      // keys 64c .. 64c+63 into columns 32c .. 32c+31, all of them S columns
      // this thread has already read
      tmem_st32(sa + 32u * c, pk);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(p_full0 + 8u * b);  // P_g(j) and the O rescale (tcgen05.st) are complete
    const unsigned long long s2 = add_f2(add_f2(sumv[0], sumv[1]), add_f2(sumv[2], sumv[3]));
    float sa2, sb2;
    f2_split(s2, sa2, sb2);
    const float sum = sa2 + sb2;
    l = fmaf(l, alpha, sum);
    m = m_new;
  }
  float o[64];
  bool have = false;
  if (ok && nk > 0 && wait_warp(o_done, (nk - 1) & 1)) {
    tc_fence_after();
    tmem_ld64(oa, o);
    have = true;
  }
  if (qrow < tile.q1) {
    const float inv = (have && l > 0.f) ? 1.f / l : 0.f;
    T* dst = static_cast<T*>(p.out) + (static_cast<int64_t>(qrow) * p.heads + h) * kAttnD;
#pragma unroll
    for (int c = 0; c < kAttnD / 8; ++c) {
      uint32_t w4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        w4[k] = have ? pack2<T>(o[8 * c + 2 * k] * inv, o[8 * c + 2 * k + 1] * inv) : 0u;
      reinterpret_cast<uint4*>(dst)[c] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kAttnThreads, 1)
    k_attn_fwd(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 24);
  const uint32_t bar0 = smem_u32(bars);
  // barriers: q_full, kv_full[4], kv_empty[4], s_full[3] and p_full[3] (one
  // per S buffer), o_done[2] (one per group: its P V products done), done
  const uint32_t q_full = bar0;
  const uint32_t kv_full0 = bar0 + 8, kv_empty0 = kv_full0 + 8 * kAttnStages;
  const uint32_t s_full0 = kv_empty0 + 8 * kAttnStages, p_full0 = s_full0 + 8 * kSBufs;
  const uint32_t o_done0 = p_full0 + 8 * kSBufs, done_bar = o_done0 + 16;
  // the last key tile's V landed (MMA -> warp 2) / its rows past the
  // sequence end are zeroed (warp 2 -> MMA)
  const uint32_t v_req = done_bar + 8, v_fixed = done_bar + 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const AttnTile tile = p.tiles[blockIdx.x];
  const int h = blockIdx.y;
  const int nk = (tile.k1 - tile.k0 + kAttnTile - 1) / kAttnTile;  // key tiles (0: empty key sequence)
  const int ngroups = tile.q0 + kAttnTile < tile.q1 ? 2 : 1;       // the second group may have no rows
  const bool last_partial = nk > 0 && tile.k1 - tile.k0 < nk * kAttnTile;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int st = 0; st < kAttnStages; ++st) {
      mbar_init(kv_full0 + 8 * st, 1);
      mbar_init(kv_empty0 + 8 * st, 1);
    }
    for (int sb = 0; sb < kSBufs; ++sb) {
      mbar_init(s_full0 + 8 * sb, 1);
      mbar_init(p_full0 + 8 * sb, 4);  // one arrival per softmax warp
    }
    mbar_init(o_done0, 1);
    mbar_init(o_done0 + 8, 1);
    mbar_init(done_bar, 1);
    mbar_init(v_req, 1);
    mbar_init(v_fixed, 1);
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
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, ngroups * kTileBytes);
      for (int g = 0; g < ngroups; ++g)
        tma_load_3d(sbase + kOffQ + g * kTileBytes, &tmQ, 0, h, tile.q0 + g * kAttnTile, q_full);
      for (int j = 0; j < nk; ++j) {
        const int st = j % kAttnStages, n = j / kAttnStages;
        if (!mbar_wait(kv_empty0 + 8 * st, (n & 1) ^ 1, p.err)) break;
        const uint32_t kb = sbase + kOffKV + st * 2 * kTileBytes;
        mbar_arrive_expect_tx(kv_full0 + 8 * st, 2 * kTileBytes);
        tma_load_3d(kb, &tmK, 0, h, tile.k0 + j * kAttnTile, kv_full0 + 8 * st);
        // V as stored: [128 keys][64 dims], read by the MMA as an MN-major operand
        tma_load_3d(kb + kTileBytes, &tmV, 0, h, tile.k0 + j * kAttnTile, kv_full0 + 8 * st);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    // Steps i = j * groups + g in order: P V of step i as soon as its P is
    // written, then S of step i + 3 into the buffer that step i's P occupied
    // once that product is done (S of the first three steps up front).  A
    // group thus usually finds its next S computed while it still works on
    // the current tile, and the tensor core alternates between the groups.
    if (lane == 0 && nk > 0) {
      const bool bf16 = std::is_same_v<T, __nv_bfloat16>;
      // P V takes V MN-major (bit 16 of the instruction descriptor): the tile
      // as TMA lands it, key rows of 64 dims in the 128-byte swizzle
      const uint32_t id_s = idesc_f16(128, 128, bf16), id_u = idesc_f16(128, 64, bf16) | (1u << 16);
      auto issue_s = [&](int step) {  // S of step into buffer step % 3; its K landed, the buffer is free
        const int g = step % ngroups, j = step / ngroups, sb = step % kSBufs;
        const uint32_t kb = sbase + kOffKV + (j % kAttnStages) * 2 * kTileBytes;
        const uint32_t qb = sbase + kOffQ + g * kTileBytes;
#pragma unroll
        for (int k = 0; k < kAttnD / 16; ++k)
          tc_mma_f16(tmem + 128u * sb, smem_desc(qb + 32u * k, 1024, 2), smem_desc(kb + 32u * k, 1024, 2), id_s,
                     k > 0 ? 1u : 0u);
        tc_commit(s_full0 + 8u * sb);
      };
      auto issue_pv = [&](int step) {  // O_g (+)= P V_j, P in the first 64 columns of buffer step % 3
        const int g = step % ngroups, j = step / ngroups, sb = step % kSBufs;
        const uint32_t vb = sbase + kOffKV + (j % kAttnStages) * 2 * kTileBytes + kTileBytes;
        // MN-major, 128B swizzle: one 64-element atom along N, 8-key groups
        // 1024 bytes apart along K; step k starts at key 16k
#pragma unroll
        for (int k = 0; k < kAttnTile / 16; ++k)
          tc_mma_f16_tmem_a(tmem + 384u + g * 64, tmem + 128u * sb + 8u * k, smem_desc(vb + 2048u * k, 1024, 2),
                            id_u, (j > 0 || k > 0) ? 1u : 0u);
        tc_commit(o_done0 + 8u * g);
      };
      auto k_landed = [&](int j) {
        const bool r = mbar_wait(kv_full0 + 8 * (j % kAttnStages), (j / kAttnStages) & 1, p.err);
        if (r && j == nk - 1 && last_partial) mbar_arrive(v_req);  // warp 2 may clear its V tail
        return r;
      };
      const int total = nk * ngroups;
      bool ok = mbar_wait(q_full, 0, p.err);
      for (int i = 0; ok && i < kSBufs && i < total; ++i) {
        if (i % ngroups == 0) ok = k_landed(i / ngroups);
        if (!ok) break;
        tc_fence_after();
        issue_s(i);
      }
      for (int i = 0; ok && i < total; ++i) {
        const int g = i % ngroups, j = i / ngroups;
        ok = mbar_wait(p_full0 + 8u * (i % kSBufs), (i / kSBufs) & 1, p.err);  // P of step i written
        if (!ok) break;
        tc_fence_after();
        if (g == 0 && j == nk - 1 && last_partial) {
          ok = mbar_wait(v_fixed, 0, p.err);  // warp 2 cleared the V rows past the sequence end
          if (!ok) break;
          tc_fence_after();
        }
        issue_pv(i);
        if (g == ngroups - 1) tc_commit(kv_empty0 + 8 * (j % kAttnStages));  // K_j and V_j are no longer read
        const int i3 = i + kSBufs;
        if (i3 < total) {
          if (i3 % ngroups == 0) ok = k_landed(i3 / ngroups);
          ok = ok && mbar_wait(o_done0 + 8u * g, j & 1, p.err);  // P V of step i done: its buffer is free
          if (!ok) break;
          tc_fence_after();
          issue_s(i3);
        }
      }
      // every MMA issued must finish before TMEM is released
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, p.err);
    }
  } else if (warp == 2) {
    // ------------------------------------------------- V tail of the last tile
    // The last key tile of a sequence also holds rows of the next sequence
    // (or TMA zero fill) past its end.  Their weights are 0, but 0 * NaN is
    // NaN: those V rows are zeroed in shared memory before the tile's first
    // P V, so one sequence's values never reach another's output (K rows
    // there are harmless: their scores are masked).
    if (last_partial) {
      int w = 1;
      if (lane == 0) w = mbar_wait(v_req, 0, p.err) ? 1 : 0;
      if (__shfl_sync(0xffffffffu, w, 0) != 0) {
        const int valid = tile.k1 - (tile.k0 + (nk - 1) * kAttnTile);
        const uint32_t vb = sbase + kOffKV + ((nk - 1) % kAttnStages) * 2 * kTileBytes + kTileBytes;
        for (uint32_t a = vb + 128u * valid + 16u * lane; a < vb + kTileBytes; a += 512u)
          asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0u) : "memory");
        fence_proxy_async_smem();  // the generic stores before the MMA's async-proxy reads
        __syncwarp();
        if (lane == 0) mbar_arrive(v_fixed);
      }
    }
  } else if (warp >= 4 && (warp - 4) / 4 < ngroups) {
    // ------------------------------------------------------------ softmax
    const int g = (warp - 4) / 4;
    softmax_group<T>(p, tile, h, nk, g, ngroups, warp & 3, lane, tmem, s_full0, p_full0, o_done0 + 8u * g);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T>
sc_status launch_attn(Handle* h, const void* q, const void* k, const void* v, void* out, const int32_t* cu_q,
                      const int32_t* cu_kv, int batch, int heads, float scale) {
  const bool bf16 = std::is_same_v<T, __nv_bfloat16>;
  const int64_t nq = cu_q[batch], nkv = cu_kv[batch];
  // host plan: one tile per 256 query rows of a sequence
  std::vector<AttnTile> tiles;
  for (int b = 0; b < batch; ++b)
    for (int32_t q0 = cu_q[b]; q0 < cu_q[b + 1]; q0 += 2 * kAttnTile)
      tiles.push_back(AttnTile{q0, cu_q[b + 1], cu_kv[b], cu_kv[b + 1], 0, 0});
  if (tiles.empty()) return SC_OK;
  const size_t tile_bytes = sizeof(AttnTile) * tiles.size();
  AttnTile* d_tiles = nullptr;
  cudaError_t e = dev_alloc(h, reinterpret_cast<void**>(&d_tiles), tile_bytes);
  if (e != cudaSuccess) return cuda_error(h, e, "attention plan buffer");
  auto fail = [&](cudaError_t err, const char* what) {
    dev_free(h, d_tiles);
    return cuda_error(h, err, what);
  };
  e = cudaMemcpyAsync(d_tiles, tiles.data(), tile_bytes, cudaMemcpyHostToDevice, h->stream);
  if (e != cudaSuccess) return fail(e, "attention plan copy");
  // Q, K and V as given: [tokens, H, 64], boxes of 128 rows of one head
  CUtensorMap tq, tk, tv;
  const uint64_t row = static_cast<uint64_t>(heads) * kAttnD * 2;
  const uint64_t dq[3] = {kAttnD, static_cast<uint64_t>(heads), static_cast<uint64_t>(std::max<int64_t>(nq, 1))};
  const uint64_t dk[3] = {kAttnD, static_cast<uint64_t>(heads), static_cast<uint64_t>(std::max<int64_t>(nkv, 1))};
  const uint64_t sq[2] = {kAttnD * 2, row};
  const uint32_t bq[3] = {kAttnD, 1, kAttnTile};
  if (!make_map_3d(&tq, bf16, q, dq, sq, bq) || !make_map_3d(&tk, bf16, k, dk, sq, bq) ||
      !make_map_3d(&tv, bf16, v, dk, sq, bq)) {
    dev_free(h, d_tiles);
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
  dev_free(h, d_tiles);  // stream-ordered: released after the kernel that uses it
  return e == cudaSuccess ? SC_OK : cuda_error(h, e, "attention launch");
}

}  // namespace

sc_status attention_varlen(Handle* h, const void* q, const void* k, const void* v, void* out, const int32_t* cu_q,
                           const int32_t* cu_kv, int batch, int heads, float scale, sc_dtype dtype) {
  if (dtype == SC_BF16) return launch_attn<__nv_bfloat16>(h, q, k, v, out, cu_q, cu_kv, batch, heads, scale);
  return launch_attn<__half>(h, q, k, v, out, cu_q, cu_kv, batch, heads, scale);
}

}  // namespace sc
