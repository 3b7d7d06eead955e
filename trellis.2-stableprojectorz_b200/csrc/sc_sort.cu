// LSD radix sort of (key, uint32 value) pairs, one-sweep style (the single
// histogram pass plus one decoupled look-back pass per digit of A. Adinets and
// D. Merrill, "Onesweep: A Faster Least Significant Digit Radix Sort for GPUs",
// 2022; the look-back follows D. Merrill and M. Garland, "Single-pass Parallel
// Prefix Scan with Decoupled Look-back", 2016).
//
// One histogram kernel counts the digits of every pass in a single read of
// the keys; each pass is then ONE kernel that ranks a 2048-key tile in shared
// memory (warp match-any ranking, stable), obtains the tile's global digit
// offsets by decoupled look-back over the tiles before it, and scatters keys
// and values through shared memory so that each digit run is written
// contiguously.  Tile ids come from an atomic counter, so a tile only waits on
// tiles that have already started; every wait is bounded by kWaitLimitNs.
//
// This replaces the torch.sort of hashmap_fallback.py (README.md:111) for the
// engine's own uses: ordering output rows by neighbour mask, ordering
// down-sample parents by packed key, and the sort-mode neighbour map.
#include "sc_common.cuh"
#include "sc_internal.h"

#include <algorithm>
#include <utility>

namespace sc {
namespace {

constexpr int kRsThreads = 256;
constexpr int kRsWarps = kRsThreads / 32;
constexpr int kRsItems = 8;
constexpr int kRsTile = kRsThreads * kRsItems;  // 2048 keys per tile
constexpr int kRsBins = 256;
constexpr int kRsMaxPasses = 8;
constexpr uint32_t kFlagAgg = 1u << 30;
constexpr uint32_t kFlagPrefix = 2u << 30;
constexpr uint32_t kValMask = (1u << 30) - 1u;

__device__ __forceinline__ uint32_t digit_mask(int shift, int end_bit) {
  const int bits = min(8, end_bit - shift);
  return (1u << bits) - 1u;
}

template <typename K>
__global__ void __launch_bounds__(kRsThreads) rs_hist_kernel(const K* __restrict__ keys, int64_t n, int begin_bit,
                                                             int end_bit, int passes, uint32_t* __restrict__ ghist) {
  __shared__ uint32_t h[kRsMaxPasses][kRsBins];
  for (int i = threadIdx.x; i < kRsMaxPasses * kRsBins; i += kRsThreads) (&h[0][0])[i] = 0;
  __syncthreads();
  for (int64_t i = blockIdx.x * (int64_t)kRsThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kRsThreads) {
    const K k = keys[i];
    for (int p = 0; p < passes; ++p) {
      const int sh = begin_bit + 8 * p;
      atomicAdd(&h[p][static_cast<uint32_t>(k >> sh) & digit_mask(sh, end_bit)], 1u);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < passes * kRsBins; i += kRsThreads) {
    const uint32_t c = (&h[0][0])[i];
    if (c) atomicAdd(&ghist[i], c);
  }
}

// Exclusive scan of one value per thread across the 256-thread block.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t x, uint32_t* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) s_warp[warp] = inc;
  __syncthreads();
  uint32_t pre = 0;
#pragma unroll
  for (int w = 0; w < kRsWarps; ++w) pre += (w < warp) ? s_warp[w] : 0u;
  __syncthreads();
  return pre + inc - x;
}

template <typename K>
__global__ void __launch_bounds__(kRsThreads) rs_onesweep_kernel(const K* __restrict__ kin,
                                                                 const uint32_t* __restrict__ vin,
                                                                 K* __restrict__ kout, uint32_t* __restrict__ vout,
                                                                 int64_t n, int shift, int end_bit,
                                                                 const uint32_t* __restrict__ ghist,
                                                                 uint32_t* status, uint32_t* tile_counter, int* err) {
  __shared__ uint32_t s_tile;
  __shared__ uint32_t s_whist[kRsWarps][kRsBins + 1];
  __shared__ uint32_t s_start[kRsBins];
  __shared__ uint32_t s_gofs[kRsBins];
  __shared__ uint32_t s_warp[kRsWarps];
  __shared__ K s_keys[kRsTile];
  __shared__ uint32_t s_vals[kRsTile];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t dmask = digit_mask(shift, end_bit);
  if (tid == 0) s_tile = atomicAdd(tile_counter, 1u);
  for (int i = tid; i < kRsWarps * (kRsBins + 1); i += kRsThreads) (&s_whist[0][0])[i] = 0;
  __syncthreads();
  const uint32_t tile = s_tile;
  const int64_t base = static_cast<int64_t>(tile) * kRsTile;

  K k[kRsItems];
  uint32_t v[kRsItems], d[kRsItems], r[kRsItems];
#pragma unroll
  for (int j = 0; j < kRsItems; ++j) {
    const int64_t idx = base + warp * (32 * kRsItems) + j * 32 + lane;
    const bool ok = idx < n;
    k[j] = ok ? kin[idx] : K(0);
    v[j] = ok ? vin[idx] : 0u;
    d[j] = ok ? (static_cast<uint32_t>(k[j] >> shift) & dmask) : static_cast<uint32_t>(kRsBins);
  }
  // Stable rank within the warp: slot by slot, peers with equal digits.
  const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
  for (int j = 0; j < kRsItems; ++j) {
    const uint32_t peers = __match_any_sync(0xffffffffu, d[j]);
    const uint32_t b = s_whist[warp][d[j]];
    r[j] = b + __popc(peers & lt);
    __syncwarp();
    if (lane == __ffs(peers) - 1) s_whist[warp][d[j]] = b + __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // Thread `tid` owns digit `tid`: per-warp exclusive offsets and tile count.
  uint32_t cnt = 0;
#pragma unroll
  for (int w = 0; w < kRsWarps; ++w) {
    const uint32_t c = s_whist[w][tid];
    s_whist[w][tid] = cnt;
    cnt += c;
  }
  volatile uint32_t* st = status + static_cast<size_t>(tile) * kRsBins;
  st[tid] = (tile == 0 ? kFlagPrefix : kFlagAgg) | cnt;

  // Global start of this digit's bin and this tile's local digit start.
  const uint32_t binbase = block_excl_scan(ghist[tid], s_warp);
  const uint32_t start = block_excl_scan(cnt, s_warp);

  // Decoupled look-back: sum the counts of earlier tiles for digit `tid`.
  uint32_t excl = 0;
  if (tile > 0) {
    int64_t pt = static_cast<int64_t>(tile) - 1;
    unsigned long long t0 = 0;
    bool waiting = false;
    while (pt >= 0) {
      const uint32_t s = reinterpret_cast<volatile uint32_t*>(status)[static_cast<size_t>(pt) * kRsBins + tid];
      if ((s & ~kValMask) == 0u) {
        if (!waiting) {
          t0 = globaltimer_ns();
          waiting = true;
        } else if (globaltimer_ns() - t0 > kWaitLimitNs) {
          record_error(err, SC_ETIMEOUT);
          break;
        }
        __nanosleep(32);
        continue;
      }
      waiting = false;
      excl += s & kValMask;
      if (s & kFlagPrefix) break;
      --pt;
    }
    st[tid] = kFlagPrefix | (excl + cnt);
  }
  s_start[tid] = start;
  s_gofs[tid] = binbase + excl - start;  // modular: + local position >= start
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kRsItems; ++j) {
    if (d[j] < static_cast<uint32_t>(kRsBins)) {
      const uint32_t pos = s_start[d[j]] + s_whist[warp][d[j]] + r[j];
      s_keys[pos] = k[j];
      s_vals[pos] = v[j];
    }
  }
  __syncthreads();
  const int tile_n = static_cast<int>(min(static_cast<int64_t>(kRsTile), n - base));
  for (int s = tid; s < tile_n; s += kRsThreads) {
    const K kk = s_keys[s];
    const uint32_t g = s_gofs[static_cast<uint32_t>(kk >> shift) & dmask] + static_cast<uint32_t>(s);
    kout[g] = kk;
    vout[g] = s_vals[s];
  }
}

template <typename K>
sc_status radix_sort_impl(Handle* h, K* keys, uint32_t* vals, K* keys_alt, uint32_t* vals_alt, int64_t n,
                          int begin_bit, int end_bit, void* temp, size_t temp_bytes, int* err, bool* in_alt,
                          bool hist_ready) {
  *in_alt = false;
  const int passes = (end_bit - begin_bit + 7) / 8;
  if (n <= 0 || passes <= 0) return SC_OK;
  if (passes > kRsMaxPasses || n >= static_cast<int64_t>(kValMask))
    return set_error(h, SC_EINVAL, "radix sort: too many passes or keys");
  const size_t need = radix_sort_temp_bytes(n, static_cast<int>(sizeof(K)), passes);
  if (temp_bytes < need) return set_error(h, SC_EINVAL, "radix sort: temp buffer too small");
  const int64_t ntiles = (n + kRsTile - 1) / kRsTile;
  uint32_t* ghist = static_cast<uint32_t*>(temp);
  uint32_t* counters = ghist + passes * kRsBins;
  uint32_t* status = counters + 64;
  cudaError_t e = cudaSuccess;
  if (!hist_ready) {
    e = cudaMemsetAsync(temp, 0, need, h->stream);
    if (e != cudaSuccess) return cuda_error(h, e, "radix sort memset");
    const int hgrid = static_cast<int>(std::min<int64_t>(ntiles, static_cast<int64_t>(h->num_sms) * 4));
    ++h->launches;
    rs_hist_kernel<K><<<hgrid, kRsThreads, 0, h->stream>>>(keys, n, begin_bit, end_bit, passes, ghist);
  }
  K* ksrc = keys;
  K* kdst = keys_alt;
  uint32_t* vsrc = vals;
  uint32_t* vdst = vals_alt;
  for (int p = 0; p < passes; ++p) {
    ++h->launches;
    rs_onesweep_kernel<K><<<static_cast<unsigned>(ntiles), kRsThreads, 0, h->stream>>>(
        ksrc, vsrc, kdst, vdst, n, begin_bit + 8 * p, end_bit, ghist + p * kRsBins,
        status + static_cast<size_t>(p) * ntiles * kRsBins, counters + p, err);
    std::swap(ksrc, kdst);
    std::swap(vsrc, vdst);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(h, e, "radix sort launch");
  *in_alt = (passes & 1) != 0;
  return SC_OK;
}

}  // namespace

size_t radix_sort_temp_bytes(int64_t n, int /*key_bytes*/, int passes) {
  const int64_t ntiles = (n + kRsTile - 1) / kRsTile;
  return sizeof(uint32_t) * (static_cast<size_t>(passes) * kRsBins + 64 +
                             static_cast<size_t>(passes) * static_cast<size_t>(ntiles) * kRsBins);
}

sc_status radix_sort_pairs_u64(Handle* h, uint64_t* keys, uint32_t* vals, uint64_t* keys_alt, uint32_t* vals_alt,
                               int64_t n, int begin_bit, int end_bit, void* temp, size_t temp_bytes, int* err,
                               bool* in_alt) {
  return radix_sort_impl<unsigned long long>(h, reinterpret_cast<unsigned long long*>(keys), vals,
                                             reinterpret_cast<unsigned long long*>(keys_alt), vals_alt, n, begin_bit,
                                             end_bit, temp, temp_bytes, err, in_alt, false);
}

sc_status radix_sort_pairs_u32(Handle* h, uint32_t* keys, uint32_t* vals, uint32_t* keys_alt, uint32_t* vals_alt,
                               int64_t n, int begin_bit, int end_bit, void* temp, size_t temp_bytes, int* err,
                               bool* in_alt, bool hist_ready) {
  return radix_sort_impl<uint32_t>(h, keys, vals, keys_alt, vals_alt, n, begin_bit, end_bit, temp, temp_bytes, err,
                                   in_alt, hist_ready);
}

}  // namespace sc
