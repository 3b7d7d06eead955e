// Fused sparse conv on tcgen05 tensor cores (bf16/f16 in, f32 accumulate).
//
// Implicit GEMM over the kernel map: for each 128-row output tile and each
// neighbour offset v present in the tile,
//     D[128, bn] += gather(feats, gidx[t][v])[128, Ci] . W[:, v, :]^T
// The gathered rows arrive by TMA row gathers (tile::gather4: four rows of
// one K chunk per instruction, rows of -1 read as zeros) straight into the
// 128B/64B/32B-swizzled K-major layout the MMA reads; W[:, v, kc] arrives by
// a tiled TMA load into the same stage, and the stage completes by
// transaction count.  tcgen05.mma reads both operands from shared memory and
// accumulates in TMEM (two buffers, so the epilogue of one tile group
// overlaps the main loop of the next).  The epilogue adds bias and
// optionally LayerNorm / SiLU / residual and stores bf16/f16 rows.
//
// Warp roles (416 threads, one persistent CTA per SM):
//   warps 0-7  producers in two groups of four taking alternate (K chunk,
//              offset) stages; within a group each lane issues one gather4
//              per stage, quads with no row are zero-filled instead; the
//              group leader also loads the weight tile
//   warp 8     TMEM allocator + single-thread MMA issuer
//   warps 9-12 epilogue (warp w reads TMEM lanes 32*(w%4) .. +31)
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
  const void* feats;
  const void* bias;
  const void* residual;
  void* out;
  const int32_t* group_order;  // groups by descending work (null: natural order)
  int64_t num_items;  // tile groups * co_blocks
  int64_t num_tiles;
  int co_blocks;
  int K;
  int ci;
  int co;
  int bn;       // output channels per item (MMA N)
  int nchunks;  // ci / KC
  uint32_t epi;
  float eps;
  int* err;
  // Halo exchange to wait for (null flags: none).  Groups ending past
  // wait_tile gather halo rows: a producer warp waits for the exchange before
  // its first such group, and at the latest before it exits.
  const uint32_t* wait_flags;
  int64_t wait_tile;
  uint32_t wait_epoch;
  int wait_world;
  int wait_rank;
};

// Warp-wide bounded wait for a halo exchange: lane r polls word r of `flags`
// (r < world, r != rank) with system-scope acquire loads until it reaches
// `epoch` (wrap-safe), then the warp synchronises, so every lane's later loads
// see the rows the peers stored before publishing.  Gives up after half the
// pipeline wait limit with SC_ETIMEOUT, so a late exchange never lets the
// conv's own stage waits (started no earlier) run out first.
constexpr unsigned long long kHaloFlagLimitNs = kWaitLimitNs / 2;
__device__ __forceinline__ void halo_flags_wait_warp(const uint32_t* flags, int world, int rank, uint32_t epoch,
                                                     int* err) {
  const int r = threadIdx.x & 31;
  if (r < world && r != rank) {
    const unsigned long long t0 = globaltimer_ns();
    unsigned ns = 32;
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
      if (static_cast<int32_t>(v - epoch) >= 0) break;
      if (globaltimer_ns() - t0 > kHaloFlagLimitNs) {
        record_error(err, SC_ETIMEOUT);
        break;
      }
      __nanosleep(ns);
      if (ns < 256) ns <<= 1;
    }
  }
  __syncwarp();
}

constexpr int kGroupWarps = 4;     // producer warps per group (one per SM sub-partition)
constexpr int kGroups = 2;         // producer groups, taking alternate stages
constexpr int kProducerWarps = kGroupWarps * kGroups;  // warps 0-7
constexpr int kMmaWarp = 8;
constexpr int kEpiWarp0 = 9;       // warps 9-12: epilogue
constexpr int kIdxAhead = 4;  // stages whose gather indices a producer warp holds in registers
constexpr int kTcThreads = (kEpiWarp0 + 4) * 32;

// Shared-memory plan for one CTA.  A stage holds TPI gathered A tiles
// (128 rows x KC each) and one weight tile (BNMAX rows x KC) that all TPI
// tiles multiply, so weight traffic per output row drops by TPI.
template <int KC, int BNMAX, int TPI>
struct TcShape {
  static constexpr int kABytes = 128 * KC * 2;  // one tile's A operand
  static constexpr int kBBytes = BNMAX * KC * 2;
  static constexpr int kStageBytes = TPI * kABytes + kBBytes;
  static constexpr int kOutBytes = 4 * 32 * 16 * 2;  // epilogue staging: per warp 32 rows x 16 columns
  static constexpr int kBarBytesPlan = 256, kAlignSlack = 1024;
  static constexpr int kStageBudget = 227 * 1024 - kOutBytes - kBarBytesPlan - kAlignSlack;
  static constexpr int kStagesFit = kStageBudget / kStageBytes;
  // an even count, so each of the two producer groups owns half the slots
  static constexpr int kStages = (kStagesFit > 12 ? 12 : kStagesFit) & ~1;
  static_assert(kStages >= 4, "not enough shared memory for four stages");
  static constexpr int kAccCols = TPI * BNMAX;  // TMEM columns of one accumulator buffer
  static constexpr uint32_t kTmemCols =
      (2 * kAccCols <= 32) ? 32 : (2 * kAccCols <= 64) ? 64 : (2 * kAccCols <= 128) ? 128 : (2 * kAccCols <= 256) ? 256 : 512;
  static_assert(2 * kAccCols <= 512, "two accumulator buffers must fit in TMEM");
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = kStages * kStageBytes + kOutBytes + kBarBytes + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory plan too large");
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
  // uniform tests once per chunk (per-element tests of the bias pointer kept
  // its loads behind a branch each)
  if (!live) {
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = 0.f;
  }
  if (bias) {
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] += Cvt<T>::to_f(bias[col0 + c0 + j]);
  }
  float s = 0.f;
  if (sq) {
#pragma unroll
    for (int j = 0; j < W; ++j) s += (v[j] - shift) * (v[j] - shift);
  } else {
#pragma unroll
    for (int j = 0; j < W; ++j) s += v[j] - shift;
  }
  return s;
}

// Epilogue of W columns (32 or 16) of the warp's 32 output rows: +bias,
// LayerNorm, SiLU, +residual, bf16/f16 pack, then a store through the warp's
// shared-memory buffer so each store instruction covers whole 32-byte row
// segments of 16 rows instead of 16 bytes of 32 rows.
template <typename T, int W>
__device__ __forceinline__ void epi_chunk(uint32_t tb, int c0, bool live, const T* bias, const T* res, T* out,
                                          int r, int co, int col0, float mean, float rstd, uint32_t epi,
                                          uint8_t* wbuf, int lane) {
  float v[W];
  tmem_ld<W>(tb + c0, v);
  // Flags and the bias are uniform across the warp: test them once per chunk.
  // Tested per element, the bias pointer kept each bias load behind its own
  // branch and the epilogue ran 2.5-3x slower (512^3 down conv 0.26 ->
  // 0.11 ms).
  if (!live) {
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = 0.f;
  }
  if (bias) {
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] += Cvt<T>::to_f(bias[col0 + c0 + j]);
  }
  if (epi & SC_EPI_LAYERNORM) {
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = (v[j] - mean) * rstd;
  }
  if (epi & SC_EPI_SILU) {
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = silu_f(v[j]);
  }
  if ((epi & SC_EPI_RESIDUAL) && r >= 0) {
    float rr[W];
    load_row<T, W>(res + static_cast<int64_t>(r) * co + col0 + c0, rr);
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] += rr[j];
  }
  // Pack and store in 16-column halves: each lane writes its row's 32-byte
  // half-segment to the warp's buffer (two 16-byte chunks, XOR-swizzled by
  // row pair), then each store instruction writes the half-segments of 16 rows.
#pragma unroll
  for (int hlf = 0; hlf < W / 16; ++hlf) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint32_t w4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = v[hlf * 16 + q * 8 + 2 * j], b = v[hlf * 16 + q * 8 + 2 * j + 1];
        if constexpr (std::is_same_v<T, __nv_bfloat16>) {
          const __nv_bfloat162 bb = __floats2bfloat162_rn(a, b);
          w4[j] = *reinterpret_cast<const uint32_t*>(&bb);
        } else {
          const __half2 bb = __floats2half2_rn(a, b);
          w4[j] = *reinterpret_cast<const uint32_t*>(&bb);
        }
      }
      *reinterpret_cast<uint4*>(wbuf + lane * 32 + ((q ^ ((lane >> 2) & 1)) * 16)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int lr = i * 16 + lane / 2;  // row within the warp
      const int ch = lane & 1;
      const int orow = __shfl_sync(0xffffffffu, r, lr);
      const uint4 val = *reinterpret_cast<const uint4*>(wbuf + lr * 32 + ((ch ^ ((lr >> 2) & 1)) * 16));
      if (orow >= 0)
        *reinterpret_cast<uint4*>(out + static_cast<int64_t>(orow) * co + col0 + c0 + hlf * 16 + ch * 8) = val;
    }
    __syncwarp();
  }
}

template <int KC, int BNMAX, int TPI, bool BF16, bool WAIT>
__global__ void __launch_bounds__(kTcThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmF, const TcParams p) {
  using S = TcShape<KC, BNMAX, TPI>;
  using Z = SwizzleCfg<KC>;
  using T = std::conditional_t<BF16, __nv_bfloat16, __half>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* out_s = smem + S::kStages * S::kStageBytes;  // [4 warps][32 rows][16 cols]
  uint64_t* bars = reinterpret_cast<uint64_t*>(out_s + S::kOutBytes);
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
      // every warp of the stage's producer group posts its bytes with one
      // arrival; its TMA copies complete them
      mbar_init(full0 + 8u * s, kGroupWarps);
      mbar_init(empty0 + 8u * s, 1);
    }
    mbar_init(tfull0, 1);
    mbar_init(tfull0 + 8u, 1);
    mbar_init(tempty0, 128);
    mbar_init(tempty0 + 8u, 128);
    mbar_init(done_bar, 1);
    fence_mbar_init();
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmF);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(s_tmem), S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int bn = p.bn;
  // An item is a group of TPI consecutive tiles times one block of bn output
  // channels; the group runs the union of its tiles' offsets.  Items are taken
  // in the map's work order (groups by descending offset count) in rounds of
  // gridDim.x, this CTA taking position blockIdx.x of even rounds and
  // gridDim.x-1-blockIdx.x of odd rounds, so every CTA gets about the same
  // work (static striding of the natural order left the busiest CTA ~18%
  // above the mean on the 256^3 workload).  All three roles walk the same
  // sequence.
  auto next_item = [&](int64_t& r) -> int64_t {  // item of round >= r (r updated), -1 when done
    for (;; ++r) {
      if (r * static_cast<int64_t>(gridDim.x) >= p.num_items) return -1;
      const int64_t pos = (r & 1) ? static_cast<int64_t>(gridDim.x) - 1 - blockIdx.x : blockIdx.x;
      const int64_t j = r * static_cast<int64_t>(gridDim.x) + pos;
      if (j < p.num_items) return j;
    }
  };
  auto item_group = [&](int64_t j, int& cb) -> int64_t {
    const int64_t q = j / p.co_blocks;
    cb = static_cast<int>(j - q * p.co_blocks);
    return p.group_order ? static_cast<int64_t>(__ldg(p.group_order + q)) : q;
  };
  auto group_mask = [&](int64_t g) {
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < TPI; ++i)
      if (g * TPI + i < p.num_tiles) m |= __ldg(p.tile_mask + g * TPI + i);
    return m;
  };

  // The stage sequence is (item, K chunk, active offset) with K chunks
  // outermost, so every output row accumulates (chunk, offset) products in
  // the same order in every conv kernel.  Both producer groups and the MMA
  // issuer walk it; a Cursor is one position in it.
  struct Cursor {
    int64_t round, item, g;
    int cb, kc, v;
    uint32_t mask0, mask;
  };
  auto enter_item = [&](Cursor& c) {  // first stage of item >= c.round's, skipping items with no offsets
    for (c.item = next_item(c.round); c.item >= 0; ++c.round, c.item = next_item(c.round)) {
      c.g = item_group(c.item, c.cb);
      c.mask0 = group_mask(c.g);
      if (c.mask0) break;
    }
    if (c.item >= 0) {
      c.kc = 0;
      c.mask = c.mask0;
      c.v = __ffs(c.mask) - 1;
    }
  };
  auto advance = [&](Cursor& c) {
    c.mask &= c.mask - 1u;
    if (!c.mask) {
      if (++c.kc < p.nchunks) {
        c.mask = c.mask0;
      } else {
        ++c.round;
        enter_item(c);
        return;
      }
    }
    c.v = __ffs(c.mask) - 1;
  };

  if (warp < kProducerWarps) {
    // ------------------------------------------------------------ producers
    // Two groups of four warps (one per SM sub-partition) take alternate
    // stages, so group g only ever uses the ring slots of parity g: while one
    // group waits for its slot and synchronises, the other issues, keeping
    // the sub-partitions' TMA issue paths busy (one sub-partition issues a
    // gather4 only every ~80 cycles; the SM's TMA unit takes one every ~19).
    // Within a group every stage is split over the four warps: warp w owns
    // quads [w*QPW, (w+1)*QPW) of the stage's TPI*32 row quads, one per lane
    // (one gather4 = four rows of one K chunk, rows of -1 read as zeros).
    // Per stage:
    //   1. the group leader waits for the slot; a barrier reduction (OR of
    //      failures) then releases the group, so all warps agree on an abort;
    //   2. a quad with no row whose slot copy already holds zeros (the lane
    //      remembers what it last wrote there) is skipped; every other quad
    //      is gathered, an empty one as four rows of -1 (zero-filled by the
    //      TMA unit, so nothing but TMA ever writes a stage);
    //   3. each warp posts its gathers' bytes (warp 0 also the weight tile's)
    //      with one arrive.expect_tx before issuing them.
    // Each warp loads its lanes' gather indices kIdxAhead of its group's
    // stages ahead into a register ring (plain coalesced loads, no staging).
    constexpr int ROWB = KC * 2;           // bytes per gathered row
    constexpr int QB = 4 * ROWB;           // bytes per row quad
    constexpr int QPW = TPI * 32 / kGroupWarps;  // row quads per warp and stage
    const int grp = warp / kGroupWarps, gw = warp % kGroupWarps;
    const uint32_t bar_id = 1u + static_cast<uint32_t>(grp);
    const bool leader = gw == 0 && lane == 0;
    const int quad_lin = gw * QPW + lane;  // this lane's quad (valid for lane < QPW)
    const int my_tile = quad_lin >> 5, my_quad = quad_lin & 31;
    const bool issuer = lane < QPW;
    const uint32_t b_tx = static_cast<uint32_t>(bn * KC * 2);
    auto load_idx = [&](const Cursor& c) -> int4 {
      const int64_t t = c.g * TPI + my_tile;
      return issuer && t < p.num_tiles
                 ? __ldg(reinterpret_cast<const int4*>(p.gidx + (t * p.K + c.v) * kTileRows) + my_quad)
                 : make_int4(-1, -1, -1, -1);
    };
    auto step = [&](Cursor& c) {  // this group's next stage
      for (int k = 0; k < kGroups && c.item >= 0; ++k) advance(c);
    };
    Cursor cur{}, ahead{};
    enter_item(cur);
    for (int k = 0; k < grp && cur.item >= 0; ++k) advance(cur);
    ahead = cur;
    int4 ring[kIdxAhead];
#pragma unroll
    for (int d = 0; d < kIdxAhead; ++d) {
      if (ahead.item >= 0) {
        ring[d] = load_idx(ahead);
        step(ahead);
      }
    }
    int64_t sidx = grp;  // position of `cur` in the CTA's stage sequence
    uint32_t used = 0, used_par = 0;  // leader: slots with a stage issued, parity of the last issue
    uint32_t zero_held = 0;           // slots whose copy of this lane's quad holds zeros
    bool abort = false;
    bool waited = !WAIT;  // WAIT: the launch waits for a halo exchange (p.wait_flags)
    while (cur.item >= 0 && !abort) {
#pragma unroll
      for (int d = 0; d < kIdxAhead; ++d) {
        if (cur.item < 0) break;
        if (WAIT && !waited && min((cur.g + 1) * TPI, p.num_tiles) > p.wait_tile) {
          halo_flags_wait_warp(p.wait_flags, p.wait_world, p.wait_rank, p.wait_epoch, p.err);
          fence_proxy_async_global();  // the TMA reads below see the peers' rows
          waited = true;
        }
        const int stage = static_cast<int>(sidx % S::kStages);
        const uint32_t phase = static_cast<uint32_t>((sidx / S::kStages) & 1);
        const uint32_t sbase = smem_base + static_cast<uint32_t>(stage * S::kStageBytes);
        const uint32_t fb = full0 + 8u * stage;
        bool fail = false;
        if (leader) {
          fail = !mbar_wait(empty0 + 8u * stage, phase ^ 1u, p.err);
          if (!fail) {
            used |= 1u << stage;
            used_par = (used_par & ~(1u << stage)) | (phase << stage);
          }
        }
        if (named_bar_red_or(bar_id, kGroupWarps * 32, fail)) {
          abort = true;
          break;
        }
        const int4 r4 = ring[d];
        const bool empty_quad = (r4.x & r4.y & r4.z & r4.w) == -1;
        const bool issue = issuer && !(empty_quad && ((zero_held >> stage) & 1u));
        if (issuer) zero_held = empty_quad ? (zero_held | (1u << stage)) : (zero_held & ~(1u << stage));
        const uint32_t n_issue = static_cast<uint32_t>(__popc(__ballot_sync(0xffffffffu, issue)));
        if (lane == 0) {
          mbar_arrive_expect_tx(fb, n_issue * QB + (gw == 0 ? b_tx : 0u));
          if (gw == 0) tma_load_2d(sbase + TPI * S::kABytes, &tmB, cur.v * p.ci + cur.kc * KC, cur.cb * bn, fb);
        }
        __syncwarp();  // the warp's bytes are posted before any of its gathers completes
        if (issue)
          tma_gather4(sbase + my_tile * S::kABytes + my_quad * QB, &tmF, cur.kc * KC, r4.x, r4.y, r4.z, r4.w, fb);
        if (ahead.item >= 0) {
          ring[d] = load_idx(ahead);
          step(ahead);
        }
        step(cur);
        sidx += kGroups;
      }
    }
    // The kernel ends only after the exchange has arrived, also when this
    // CTA gathered no halo row: the caller's next exchange may then reuse
    // the peers' buffers.
    if (WAIT && !waited) halo_flags_wait_warp(p.wait_flags, p.wait_world, p.wait_rank, p.wait_epoch, p.err);
    if (abort && leader) {
      // Error exit: let the copies already issued into our shared memory land
      // (every stage's copies, from all warps of the group, complete one barrier).
      for (int s = 0; s < S::kStages; ++s)
        if (used & (1u << s)) mbar_wait(full0 + 8u * s, (used_par >> s) & 1u, nullptr);
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, bn, BF16);
      int stage = 0;
      uint32_t phase = 0, it = 0;
      bool ok = true;
      int64_t round = 0;
      for (int64_t item = next_item(round); ok && item >= 0; ++round, item = next_item(round), ++it) {
        int cb_unused;
        const int64_t g = item_group(item, cb_unused);
        const uint32_t acc = it & 1u, aph = (it >> 1) & 1u;
        if (!mbar_wait(tempty0 + 8u * acc, aph ^ 1u, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * static_cast<uint32_t>(S::kAccCols);
        const int nsteps = __popc(group_mask(g)) * p.nchunks;
        for (int s = 0; s < nsteps; ++s) {
          if (!mbar_wait_sleep<64>(full0 + 8u * stage, phase, p.err)) {
            ok = false;
            break;
          }
          // Every byte of the stage was written by TMA (async proxy) and is
          // counted in the full barrier's transaction bytes; the wait
          // acquires them for the MMAs, which read through the same proxy.
          tc_fence_after();
          const uint32_t a0 = smem_base + static_cast<uint32_t>(stage * S::kStageBytes);
          const uint32_t b0 = a0 + TPI * S::kABytes;
#pragma unroll
          for (int i = 0; i < TPI; ++i) {
#pragma unroll
            for (int k = 0; k < KC / 16; ++k) {
              tc_mma_f16(d_tmem + i * BNMAX, smem_desc(a0 + i * S::kABytes + 32u * k, Z::kSbo, Z::kMode),
                         smem_desc(b0 + 32u * k, Z::kSbo, Z::kMode), idesc, (s > 0 || k > 0) ? 1u : 0u);
            }
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
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const T* bias = static_cast<const T*>(p.bias);
    const T* res = static_cast<const T*>(p.residual);
    T* out = static_cast<T*>(p.out);
    uint8_t* wbuf = out_s + (warp - kEpiWarp0) * (32 * 32);
    uint32_t it = 0;
    int64_t round = 0;
    for (int64_t item = next_item(round); item >= 0; ++round, item = next_item(round), ++it) {
      int cb;
      const int64_t g = item_group(item, cb);
      const uint32_t acc = it & 1u, aph = (it >> 1) & 1u;
      int w = 1;
      if (lane == 0) w = mbar_wait_sleep(tfull0 + 8u * acc, aph, p.err) ? 1 : 0;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) break;
      tc_fence_after();
      const bool live = group_mask(g) != 0u;
      const int col0 = cb * bn;
      const int bn32 = bn & ~31;  // columns handled 32 at a time; a 16-wide tail follows when bn % 32 == 16
#pragma unroll 1
      for (int i = 0; i < TPI; ++i) {
        const int64_t t = g * TPI + i;
        const int r = t < p.num_tiles ? __ldg(p.tile_rows + t * 128 + row) : -1;
        const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                            acc * static_cast<uint32_t>(S::kAccCols) + static_cast<uint32_t>(i * BNMAX);
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
        for (int c0 = 0; c0 < bn32; c0 += 32)
          epi_chunk<T, 32>(tb, c0, live, bias, res, out, r, p.co, col0, mean, rstd, p.epi, wbuf, lane);
        if (bn32 < bn) epi_chunk<T, 16>(tb, bn32, live, bias, res, out, r, p.co, col0, mean, rstd, p.epi, wbuf, lane);
      }
      tc_fence_before();
      mbar_arrive(tempty0 + 8u * acc);
      __syncwarp();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

// ------------------------------------------------------- halo-staged conv
// For maps built with SC_BUILD_HALO (tiles = 128 consecutive output rows).
// A Morton-ordered tile's 27 x 128 gathers read only a few hundred distinct
// input rows (245 on average on the 256^3 shell workload, against 1,958
// gathered rows), so each tile's distinct rows are staged in shared memory
// once per 64-channel chunk by TMA row gathers, and the A operand of every
// offset is assembled from that halo straight into tensor memory:
//   warps 0-7  A builders in two groups of four (warp w writes TMEM lanes
//              32*(w%4)..+31); group g takes the (chunk, offset) steps with
//              step % 2 == g: each lane copies its row's 64 channels from
//              the halo (or zeros) into TMEM with tcgen05.st
//   warp 8     TMEM allocator + single-thread MMA issuer (A from TMEM, weight
//              tile B from shared memory)
//   warps 9-12 epilogue (as in conv_tc_kernel)
//   warp 13    TMA: per tile the 6.9 KB position block, per chunk the halo
//   warp 14    TMA: weight tiles per (chunk, offset)
// Products are accumulated chunk by chunk and offset by offset, the same order
// as conv_tc_kernel, so both kernels give identical results.
constexpr int kHaloKernelThreads = 480;
constexpr int kHaloMmaWarp = 8, kHaloEpiWarp0 = 9, kHaloTmaWarp = 13;
constexpr int kHaloBStages = 6;
constexpr int kHaloASlots = 8;
constexpr int kHaloSlotBytes = kHaloCap * 128;
constexpr int kLidxBytes = 27 * 128 * 2;
constexpr int kHaloBarBytes = 512;
constexpr int kHaloSmemBytes = 2 * kHaloSlotBytes + kHaloBStages * 16384 + 2 * kLidxBytes + 4096 + kHaloBarBytes + 1024;
static_assert(kHaloSmemBytes <= 227 * 1024, "halo conv shared memory plan too large");
constexpr uint32_t kHaloAccCols = 128, kHaloACol0 = 256, kHaloTmemCols = 512;

struct HaloConvParams {
  const void* feats;
  const int32_t* gidx;
  const int32_t* halo_rows;
  const int32_t* halo_n;
  const uint16_t* lidx;
  const int32_t* tile_rows;
  const uint32_t* tile_mask;
  const int32_t* group_order;
  const void* bias;
  const void* residual;
  void* out;
  int64_t num_tiles;
  int ci;
  int co;
  int nchunks;
  uint32_t epi;
  float eps;
  int* err;
};

template <bool BF16>
__global__ void __launch_bounds__(kHaloKernelThreads, 1)
    conv_halo_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmF,
                     const HaloConvParams p) {
  using T = std::conditional_t<BF16, __nv_bfloat16, __half>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* halo_s = smem;                                              // [2][kHaloCap rows][128 B], 128B-swizzled
  uint8_t* b_s = halo_s + 2 * kHaloSlotBytes;                          // [kHaloBStages][co rows][128 B]
  uint16_t* lidx_s = reinterpret_cast<uint16_t*>(b_s + kHaloBStages * 16384);  // [2][27][128]
  uint8_t* out_s = reinterpret_cast<uint8_t*>(lidx_s) + 2 * kLidxBytes;       // [4 warps][32 rows][16 cols]
  uint64_t* bars = reinterpret_cast<uint64_t*>(out_s + 4096);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 42);
  static_assert((2 * 4 + 2 * kHaloBStages + 2 * kHaloASlots + 5) * 8 + 8 <= kHaloBarBytes, "barrier area");
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t hfull0 = bar0, hempty0 = bar0 + 16, lfull0 = bar0 + 32, lempty0 = bar0 + 48;
  const uint32_t bfull0 = bar0 + 64, bempty0 = bfull0 + 8 * kHaloBStages;
  const uint32_t afull0 = bempty0 + 8 * kHaloBStages, aempty0 = afull0 + 8 * kHaloASlots;
  const uint32_t tfull0 = aempty0 + 8 * kHaloASlots, tempty0 = tfull0 + 16, done_bar = tfull0 + 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int co = p.co;
  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(hfull0 + 8u * s, 1);
      mbar_init(hempty0 + 8u * s, 8);
      mbar_init(lfull0 + 8u * s, 1);
      mbar_init(lempty0 + 8u * s, 8);
      mbar_init(tfull0 + 8u * s, 1);
      mbar_init(tempty0 + 8u * s, 128);
    }
    for (int s = 0; s < kHaloBStages; ++s) {
      mbar_init(bfull0 + 8u * s, 1);
      mbar_init(bempty0 + 8u * s, 1);
    }
    for (int s = 0; s < kHaloASlots; ++s) {
      mbar_init(afull0 + 8u * s, 4);
      mbar_init(aempty0 + 8u * s, 1);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmF);
  }
  if (warp == kHaloMmaWarp) {
    tmem_alloc(smem_u32(s_tmem), kHaloTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  // Item sequence: same serpentine rounds over the work order as conv_tc_kernel.
  auto next_item = [&](int64_t& r) -> int64_t {
    for (;; ++r) {
      if (r * static_cast<int64_t>(gridDim.x) >= p.num_tiles) return -1;
      const int64_t pos = (r & 1) ? static_cast<int64_t>(gridDim.x) - 1 - blockIdx.x : blockIdx.x;
      const int64_t j = r * static_cast<int64_t>(gridDim.x) + pos;
      if (j < p.num_tiles) return j;
    }
  };
  auto tile_of = [&](int64_t j) -> int64_t {
    return p.group_order ? static_cast<int64_t>(__ldg(p.group_order + j)) : j;
  };

  if (warp < 8) {
    // ------------------------------------------------------- A builders
    const int q = warp & 3, grp = warp >> 2;
    uint32_t lph = 0, hph = 0;
    int ls = 0, hs = 0;
    uint32_t step = 0;  // (chunk, offset) steps of this CTA so far, both groups
    bool ok = true;
    auto wait_all = [&](uint32_t bar, uint32_t par) {
      int w = 1;
      if (lane == 0) w = mbar_wait(bar, par, p.err) ? 1 : 0;
      w = __shfl_sync(0xffffffffu, w, 0);
      return w != 0;
    };
    int64_t round = 0;
    for (int64_t j = next_item(round); ok && j >= 0; ++round, j = next_item(round)) {
      const int64_t t = tile_of(j);
      const uint32_t mask0 = __ldg(p.tile_mask + t);
      // tiles with more distinct rows than a halo slot holds read their rows
      // straight from global memory (these threads issue no async copies)
      const bool direct = __ldg(p.halo_n + t) > kHaloCap;
      if (!wait_all(lfull0 + 8u * ls, lph)) { ok = false; break; }
      const uint16_t* lrow = lidx_s + ls * (27 * 128) + q * 32 + lane;
      const int32_t* grow = p.gidx + t * 27 * 128 + q * 32 + lane;
      for (int kc = 0; ok && kc < p.nchunks; ++kc) {
        if (!wait_all(hfull0 + 8u * hs, hph)) { ok = false; break; }
        const uint32_t hbase = smem_u32(halo_s + hs * kHaloSlotBytes);
        uint32_t mask = mask0;
        while (mask) {
          const int v = __ffs(mask) - 1;
          mask &= mask - 1u;
          const uint32_t my = step++;
          if ((my & 1u) != static_cast<uint32_t>(grp)) continue;
          const uint32_t as = my % kHaloASlots, aph = (my / kHaloASlots) & 1u;
          if (!wait_all(aempty0 + 8u * as, aph ^ 1u)) { ok = false; break; }
          tc_fence_after();
          uint32_t val[32];
          if (direct) {
            const int r = __ldg(grow + v * 128);
            if (r >= 0) {
              const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(p.feats) +
                                                                static_cast<int64_t>(r) * p.ci + kc * 64);
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                const uint4 u = __ldg(src + c);
                val[4 * c] = u.x;
                val[4 * c + 1] = u.y;
                val[4 * c + 2] = u.z;
                val[4 * c + 3] = u.w;
              }
            } else {
#pragma unroll
              for (int c = 0; c < 32; ++c) val[c] = 0u;
            }
          } else if (const uint32_t l = lrow[v * 128]; l != 0xFFFFu) {
            const uint32_t rb = hbase + l * 128u;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint32_t a, b, cc, d;
              asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(a), "=r"(b), "=r"(cc), "=r"(d)
                           : "r"(rb + ((static_cast<uint32_t>(c) ^ (l & 7u)) << 4)));
              val[4 * c] = a;
              val[4 * c + 1] = b;
              val[4 * c + 2] = cc;
              val[4 * c + 3] = d;
            }
          } else {
#pragma unroll
            for (int c = 0; c < 32; ++c) val[c] = 0u;
          }
          tmem_st32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + kHaloACol0 + as * 32u, val);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(afull0 + 8u * as);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(hempty0 + 8u * hs);
        if (++hs == 2) {
          hs = 0;
          hph ^= 1u;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(lempty0 + 8u * ls);
      if (++ls == 2) {
        ls = 0;
        lph ^= 1u;
      }
    }
  } else if (warp == kHaloMmaWarp) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, co, BF16);
      int bs = 0, as = 0;
      uint32_t bph = 0, aph = 0, it = 0;
      bool ok = true;
      int64_t round = 0;
      for (int64_t j = next_item(round); ok && j >= 0; ++round, j = next_item(round), ++it) {
        const int64_t t = tile_of(j);
        const uint32_t mask0 = __ldg(p.tile_mask + t);
        const uint32_t acc = it & 1u, tph = (it >> 1) & 1u;
        if (!mbar_wait(tempty0 + 8u * acc, tph ^ 1u, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kHaloAccCols;
        bool first = true;
        for (int kc = 0; ok && kc < p.nchunks; ++kc) {
          uint32_t mask = mask0;
          while (mask) {
            mask &= mask - 1u;
            if (!mbar_wait_sleep<64>(afull0 + 8u * as, aph, p.err) || !mbar_wait(bfull0 + 8u * bs, bph, p.err)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t b0 = smem_u32(b_s + bs * 16384);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc_mma_f16_tmem_a(d_tmem, tmem_base + kHaloACol0 + as * 32u + 8u * k, smem_desc(b0 + 32u * k, 1024, 2),
                                idesc, (first && k == 0) ? 0u : 1u);
            first = false;
            tc_commit(aempty0 + 8u * as);
            tc_commit(bempty0 + 8u * bs);
            if (++as == kHaloASlots) {
              as = 0;
              aph ^= 1u;
            }
            if (++bs == kHaloBStages) {
              bs = 0;
              bph ^= 1u;
            }
          }
        }
        if (!ok) break;
        tc_commit(tfull0 + 8u * acc);
      }
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, p.err);
    }
    __syncwarp();
  } else if (warp < kHaloTmaWarp) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const T* bias = static_cast<const T*>(p.bias);
    const T* res = static_cast<const T*>(p.residual);
    T* out = static_cast<T*>(p.out);
    uint8_t* wbuf = out_s + (warp - kHaloEpiWarp0) * (32 * 32);
    uint32_t it = 0;
    int64_t round = 0;
    for (int64_t j = next_item(round); j >= 0; ++round, j = next_item(round), ++it) {
      const int64_t t = tile_of(j);
      const uint32_t acc = it & 1u, aph = (it >> 1) & 1u;
      int w = 1;
      if (lane == 0) w = mbar_wait_sleep(tfull0 + 8u * acc, aph, p.err) ? 1 : 0;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) break;
      tc_fence_after();
      const bool live = __ldg(p.tile_mask + t) != 0u;
      const int bn32 = co & ~31;
      const int r = __ldg(p.tile_rows + t * 128 + row);
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kHaloAccCols;
      float mean = 0.f, rstd = 1.f;
      if (p.epi & SC_EPI_LAYERNORM) {
        float s1 = 0.f;
        for (int c0 = 0; c0 < bn32; c0 += 32) s1 += chunk_sum<T, 32>(tb, c0, live, bias, 0, 0.f, false);
        if (bn32 < co) s1 += chunk_sum<T, 16>(tb, bn32, live, bias, 0, 0.f, false);
        mean = s1 / static_cast<float>(co);
        float s2 = 0.f;
        for (int c0 = 0; c0 < bn32; c0 += 32) s2 += chunk_sum<T, 32>(tb, c0, live, bias, 0, mean, true);
        if (bn32 < co) s2 += chunk_sum<T, 16>(tb, bn32, live, bias, 0, mean, true);
        rstd = rsqrtf(s2 / static_cast<float>(co) + p.eps);
      }
      for (int c0 = 0; c0 < bn32; c0 += 32)
        epi_chunk<T, 32>(tb, c0, live, bias, res, out, r, co, 0, mean, rstd, p.epi, wbuf, lane);
      if (bn32 < co) epi_chunk<T, 16>(tb, bn32, live, bias, res, out, r, co, 0, mean, rstd, p.epi, wbuf, lane);
      tc_fence_before();
      mbar_arrive(tempty0 + 8u * acc);
      __syncwarp();
    }
  } else if (warp == kHaloTmaWarp) {
    // ------------------------------------------ TMA: positions and halos
    if (lane == 0) {
      int ls = 0, hs = 0;
      uint32_t lph = 0, hph = 0;
      uint32_t lused = 0, lpar = 0, hused = 0, hpar = 0;  // slots with a copy issued, parity of the last one
      bool ok = true;
      int64_t round = 0;
      for (int64_t j = next_item(round); ok && j >= 0; ++round, j = next_item(round)) {
        const int64_t t = tile_of(j);
        if (!mbar_wait(lempty0 + 8u * ls, lph ^ 1u, p.err)) break;
        const uint32_t lbar = lfull0 + 8u * ls;
        mbar_arrive_expect_tx(lbar, kLidxBytes);
        bulk_load(smem_u32(lidx_s + ls * (27 * 128)), p.lidx + t * (27 * 128), kLidxBytes, lbar);
        lused |= 1u << ls;
        lpar = (lpar & ~(1u << ls)) | (lph << ls);
        if (++ls == 2) {
          ls = 0;
          lph ^= 1u;
        }
        const int hn_all = __ldg(p.halo_n + t);
        const int groups = hn_all > kHaloCap ? 0 : (hn_all + 3) >> 2;  // direct tiles stage nothing
        const int4* hrows = reinterpret_cast<const int4*>(p.halo_rows + t * kHaloCap);
        for (int kc = 0; kc < p.nchunks; ++kc) {
          if (!mbar_wait(hempty0 + 8u * hs, hph ^ 1u, p.err)) {
            ok = false;
            break;
          }
          const uint32_t hbar = hfull0 + 8u * hs;
          const uint32_t hdst = smem_u32(halo_s + hs * kHaloSlotBytes);
          mbar_arrive_expect_tx(hbar, static_cast<uint32_t>(groups) * 512u);
          for (int g4 = 0; g4 < groups; ++g4) {
            const int4 r4 = __ldg(hrows + g4);
            tma_gather4(hdst + g4 * 512u, &tmF, kc * 64, r4.x, r4.y, r4.z, r4.w, hbar);
          }
          hused |= 1u << hs;
          hpar = (hpar & ~(1u << hs)) | (hph << hs);
          if (++hs == 2) {
            hs = 0;
            hph ^= 1u;
          }
        }
      }
      // Let every copy issued into this CTA's shared memory land before exit.
      for (int s = 0; s < 2; ++s) {
        if (lused & (1u << s)) mbar_wait(lfull0 + 8u * s, (lpar >> s) & 1u, nullptr);
        if (hused & (1u << s)) mbar_wait(hfull0 + 8u * s, (hpar >> s) & 1u, nullptr);
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------- TMA: weight tiles
    if (lane == 0) {
      int bs = 0;
      uint32_t bph = 0, bused = 0, bpar = 0;
      bool ok = true;
      const uint32_t b_tx = static_cast<uint32_t>(co) * 128u;
      int64_t round = 0;
      for (int64_t j = next_item(round); ok && j >= 0; ++round, j = next_item(round)) {
        const int64_t t = tile_of(j);
        const uint32_t mask0 = __ldg(p.tile_mask + t);
        for (int kc = 0; ok && kc < p.nchunks; ++kc) {
          uint32_t mask = mask0;
          while (mask) {
            const int v = __ffs(mask) - 1;
            mask &= mask - 1u;
            if (!mbar_wait(bempty0 + 8u * bs, bph ^ 1u, p.err)) {
              ok = false;
              break;
            }
            const uint32_t bbar = bfull0 + 8u * bs;
            mbar_arrive_expect_tx(bbar, b_tx);
            tma_load_2d(smem_u32(b_s + bs * 16384), &tmB, v * p.ci + kc * 64, 0, bbar);
            bused |= 1u << bs;
            bpar = (bpar & ~(1u << bs)) | (bph << bs);
            if (++bs == kHaloBStages) {
              bs = 0;
              bph ^= 1u;
            }
          }
        }
      }
      for (int s = 0; s < kHaloBStages; ++s)
        if (bused & (1u << s)) mbar_wait(bfull0 + 8u * s, (bpar >> s) & 1u, nullptr);
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kHaloMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kHaloTmemCols);
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

template <int KC, int BNMAX, int TPI, bool BF16>
sc_status launch_tc(Handle* h, const KMap* km, const void* feats, const void* weight, TcParams p) {
  using S = TcShape<KC, BNMAX, TPI>;
  using Z = SwizzleCfg<KC>;
  CUtensorMap tb, tf;
  p.feats = feats;
  // weights: [Co, K*Ci], box KC x bn; features: [n_in, Ci], box KC x 1 (row gathers)
  if (!make_map_2d(&tb, BF16, weight, static_cast<uint64_t>(km->K) * p.ci, p.co,
                   static_cast<uint64_t>(km->K) * p.ci * 2, KC, p.bn, Z::kTma) ||
      !make_map_2d(&tf, BF16, feats, p.ci, km->n_in, static_cast<uint64_t>(p.ci) * 2, KC, 1, Z::kTma))
    return set_error(h, SC_ECUDA, "cuTensorMapEncodeTiled failed");
  p.num_items = ((p.num_tiles + TPI - 1) / TPI) * p.co_blocks;
  // the wait is compiled only into launches that have one
  auto kern = p.wait_flags ? conv_tc_kernel<KC, BNMAX, TPI, BF16, true>
                           : conv_tc_kernel<KC, BNMAX, TPI, BF16, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes);
  if (e != cudaSuccess) return cuda_error(h, e, "conv smem attribute");
  const int64_t ctas = h->conv_ctas > 0 ? std::min(h->conv_ctas, h->num_sms) : h->num_sms;
  const int64_t grid = std::min<int64_t>(p.num_items, ctas);
  // Work order balances CTAs that run few items (10 per CTA on the 256^3
  // workload: -9% conv time); with many items per CTA static striding is
  // already balanced and the natural tile order keeps better L2 locality.
  p.group_order = p.num_items < kWorkOrderMaxItemsPerCta * grid ? km->group_order[TPI == 4 ? 2 : TPI - 1] : nullptr;
  ++h->launches;
  kern<<<static_cast<unsigned>(grid), kTcThreads, S::kSmemBytes, h->stream>>>(tb, tf, p);
  e = cudaGetLastError();
  return e == cudaSuccess ? SC_OK : cuda_error(h, e, "conv launch");
}

template <int KC, bool BF16>
sc_status dispatch_bn(Handle* h, const KMap* km, const void* feats, const void* weight, const TcParams& p) {
  // Up to 128 output channels two tiles share each weight stage; wider
  // outputs already reuse each gathered row across 256 MMA columns.
  // Up to 64 output channels with K chunks of at most 32 channels, four tiles
  // share each weight stage: the stages are small and their fixed cost
  // dominates (1024^3 Ci = Co = 32: 1.51 -> 1.16 ms against two tiles).
  if constexpr (KC <= 32) {
    if (p.bn <= 64) return launch_tc<KC, 64, 4, BF16>(h, km, feats, weight, p);
  }
  if (p.bn <= 64) return launch_tc<KC, 64, 2, BF16>(h, km, feats, weight, p);
  if (p.bn <= 128) return launch_tc<KC, 128, 2, BF16>(h, km, feats, weight, p);
  return launch_tc<KC, 256, 1, BF16>(h, km, feats, weight, p);
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

// 3-D tiled tensor map over 16-bit elements with the 128-byte swizzle (the
// attention kernel's Q, K and V^T tiles); strides in bytes of dims 1 and 2.
bool make_map_3d(CUtensorMap* m, bool bf16, const void* base, const uint64_t dims[3], const uint64_t strides[2],
                 const uint32_t box[3]) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  const cuuint64_t st[2] = {strides[0], strides[1]};
  const cuuint32_t bx[3] = {box[0], box[1], box[2]};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
             const_cast<void*>(base), d, st, bx, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

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
    ++h->launches;
    k_check_gidx<<<static_cast<unsigned>((total + 255) / 256), 256, 0, h->stream>>>(km->gidx, total, km->n_in, derr);
    e = cudaMemcpyAsync(&herr, derr, 4, cudaMemcpyDeviceToHost, h->stream);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  dev_free(h, derr);
  if (e != cudaSuccess) return cuda_error(h, e, "bounds check");
  if (herr) return set_error(h, SC_EINVAL, "gather index out of range");
  return SC_OK;
}


template <bool BF16>
sc_status launch_halo(Handle* h, const KMap* km, const void* feats, const void* weight, const void* bias,
                      const void* residual, void* out, int ci, int co, uint32_t epi, float eps) {
  CUtensorMap tb, tf;
  if (!make_map_2d(&tb, BF16, weight, static_cast<uint64_t>(km->K) * ci, co, static_cast<uint64_t>(km->K) * ci * 2,
                   64, co, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tf, BF16, feats, ci, km->n_in, static_cast<uint64_t>(ci) * 2, 64, 1, CU_TENSOR_MAP_SWIZZLE_128B))
    return set_error(h, SC_ECUDA, "cuTensorMapEncodeTiled failed");
  HaloConvParams p{};
  p.feats = feats;
  p.gidx = km->gidx;
  p.halo_rows = km->halo_rows;
  p.halo_n = km->halo_n;
  p.lidx = km->lidx;
  p.tile_rows = km->tile_rows;
  p.tile_mask = km->tile_mask;
  p.bias = bias;
  p.residual = residual;
  p.out = out;
  p.num_tiles = km->num_tiles;
  p.ci = ci;
  p.co = co;
  p.nchunks = ci / 64;
  p.epi = epi;
  p.eps = eps;
  p.err = h->derr;
  const int64_t ctas = h->conv_ctas > 0 ? std::min(h->conv_ctas, h->num_sms) : h->num_sms;
  const int64_t grid = std::min<int64_t>(p.num_tiles, ctas);
  p.group_order = p.num_tiles < kWorkOrderMaxItemsPerCta * grid ? km->group_order[0] : nullptr;
  auto kern = conv_halo_kernel<BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kHaloSmemBytes);
  if (e != cudaSuccess) return cuda_error(h, e, "halo conv smem attribute");
  ++h->launches;
  kern<<<static_cast<unsigned>(grid), kHaloKernelThreads, kHaloSmemBytes, h->stream>>>(tb, tf, p);
  e = cudaGetLastError();
  return e == cudaSuccess ? SC_OK : cuda_error(h, e, "halo conv launch");
}

// The halo-staged kernel applies to submanifold maps built with halo data,
// for Ci a multiple of 64 and Co <= 128.
bool halo_applies(const Handle* h, const KMap* km, int ci, int co) {
  return km->lidx && km->K == 27 && km->kind == SC_KMAP_SUBM &&
         ci % 64 == 0 && co % 16 == 0 && co >= 16 && co <= 128 && !h->debug_bounds && km->num_tiles > 0;
}

sc_status conv_tc(Handle* h, const KMap* km, const void* feats, const void* weight, const void* bias,
                  const void* residual, void* out, int ci, int co, sc_dtype dtype, uint32_t epi, float eps,
                  const ConvWait& wait) {
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
  if (halo_applies(h, km, ci, co)) {
    // the halo-staged kernel takes the exchange's wait as a separate launch
    if (wait.flags) {
      const sc_status st = halo_wait(h, wait.flags, wait.world, wait.rank, wait.epoch);
      if (st != SC_OK) return st;
    }
    return dtype == SC_BF16 ? launch_halo<true>(h, km, feats, weight, bias, residual, out, ci, co, epi, eps)
                            : launch_halo<false>(h, km, feats, weight, bias, residual, out, ci, co, epi, eps);
  }
  TcParams p{};
  p.gidx = km->gidx;
  p.tile_rows = km->tile_rows;
  p.tile_mask = km->tile_mask;
  p.bias = bias;
  p.residual = residual;
  p.out = out;
  p.co_blocks = co / bn;
  p.num_tiles = km->num_tiles;
  p.num_items = km->num_tiles * p.co_blocks;
  p.K = km->K;
  p.ci = ci;
  p.co = co;
  p.bn = bn;
  p.epi = epi;
  p.eps = eps;
  p.err = h->derr;
  if (p.num_items == 0) return wait.flags ? halo_wait(h, wait.flags, wait.world, wait.rank, wait.epoch) : SC_OK;
  // A plain map may read halo rows from its first tile; a concatenated map
  // from its second part on.
  p.wait_flags = wait.flags;
  p.wait_tile = km->split_tile >= 0 ? km->split_tile : 0;
  p.wait_epoch = wait.epoch;
  p.wait_world = wait.world;
  p.wait_rank = wait.rank;
  return dtype == SC_BF16 ? dispatch_kc<true>(h, km, feats, weight, p)
                          : dispatch_kc<false>(h, km, feats, weight, p);
}

}  // namespace sc
