// Kernel-map construction: submanifold 3x3x3 (hash or sort probe), stride-2
// down-sample and its transpose, then the tile layout the conv kernels read.
//
// Reference behaviour being replaced:
//   pass 0  src/sparse/ops/conv3d_wgsl.ts:44-71   dense sp_to_lin scatter
//   pass 1  src/sparse/ops/conv3d_wgsl.ts:75-128  27-offset neighbour lookup
//   host    src/sparse/ops/conv3d.ts:63-151        cache + dispatch
//   hashmap_fallback.py (README.md:111)            flat_idx sort + searchsorted
// The dense grid is replaced by an open-addressing hash (or a sorted key
// array); the batch index is part of every key.
#include "sc_common.cuh"
#include "sc_internal.h"

#include <algorithm>
#include <vector>

namespace sc {
namespace {

constexpr unsigned long long kEmptyKey = ~0ull;

struct __align__(16) Slot {
  unsigned long long key;
  int val;
  int pad;
};

// 16-bit fields: b | x | y | z (b <= 32767, x/y/z <= 65535, checked).
__device__ __forceinline__ unsigned long long pack16(int b, int x, int y, int z) {
  return (static_cast<unsigned long long>(b) << 48) | (static_cast<unsigned long long>(x) << 32) |
         (static_cast<unsigned long long>(y) << 16) | static_cast<unsigned long long>(z);
}

// 64-bit mixing finaliser (MurmurHash3 fmix64), folded to 32 bits.
__device__ __forceinline__ uint32_t mix64(unsigned long long k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return static_cast<uint32_t>(k);
}

// Batch index in [0, 32767] keeps the top key bit clear, so the all-ones
// empty-slot key can never collide with a voxel key.
// Probe sequence of a voxel key.  Probe 0 is the home slot: the 4x4x4 block
// containing the voxel owns a 64-slot region (hash of the block coordinates)
// and the voxel's position inside the block picks the slot, so the 27
// neighbours of a voxel start in at most eight nearby regions (cache-local).
// Probe i >= 1 is a fresh hash of (key, i): collisions leave the region instead
// of walking along it, which keeps chains as short as with a fully random hash
// (at load <= 1/4: mean 1.2 probes, p99 3 on the 256^3 shell workload).
//
// The block hash is separable: per-axis terms are multiplied by odd constants
// and xored, then finalised with a 32-bit multiply-xorshift, so a voxel's 27
// neighbours need only 3 terms per axis plus one finaliser each.  The four
// multipliers are the 32-bit primes of xxHash32 (Y. Collet, PRIME32_1..4);
// the finaliser is a two-round xorshift-multiply (shifts 15/12/15) from the
// constant search published with C. Wellons' hash-prospector.  Rehash probes
// step the key by multiples of 2^64 / golden ratio (the SplitMix64
// increment) before the MurmurHash3 fmix64 mixer.
__device__ __forceinline__ uint32_t axis_term(int v, uint32_t mul) { return static_cast<uint32_t>(v) * mul; }
constexpr uint32_t kMulB = 0x27D4EB2Fu, kMulX = 0x9E3779B1u, kMulY = 0x85EBCA77u, kMulZ = 0xC2B2AE3Du;
__device__ __forceinline__ uint32_t fin32(uint32_t h) {
  h ^= h >> 15;
  h *= 0x2C1B3C6Du;
  h ^= h >> 12;
  h *= 0x297A2D39u;
  h ^= h >> 15;
  return h;
}
__device__ __forceinline__ uint32_t local_slot(int x, int y, int z) {
  return static_cast<uint32_t>(((x & 3) << 4) | ((y & 3) << 2) | (z & 3));
}
__device__ __forceinline__ uint32_t home_slot(int b, int x, int y, int z, uint32_t cap_mask) {
  const uint32_t h = fin32(axis_term(b, kMulB) ^ axis_term(x >> 2, kMulX) ^ axis_term(y >> 2, kMulY) ^
                           axis_term(z >> 2, kMulZ));
  return ((h << 6) | local_slot(x, y, z)) & cap_mask;
}
__device__ __forceinline__ uint32_t rehash_slot(unsigned long long key, uint32_t i, uint32_t cap_mask) {
  return mix64(key ^ (static_cast<unsigned long long>(i) * 0x9E3779B97F4A7C15ull)) & cap_mask;
}

__device__ __forceinline__ bool coord_ok(int4 c) {
  return static_cast<unsigned>(c.x) <= 32767u && static_cast<unsigned>(c.y) <= 65535u &&
         static_cast<unsigned>(c.z) <= 65535u && static_cast<unsigned>(c.w) <= 65535u;
}

// Offset v = kd*9 + kh*3 + kw of a 3x3x3 kernel with per-axis dilation: kd
// on x, kh on y, kw on z (src/sparse/ops/conv3d_wgsl.ts:91-101,115-117).
__device__ __forceinline__ void offset27(int v, Dil d, int& dx, int& dy, int& dz) {
  dx = (v / 9 - 1) * d.x;
  dy = ((v / 3) % 3 - 1) * d.y;
  dz = (v % 3 - 1) * d.z;
}

// Tile rows of a concatenated map: the first map's slots, then the second
// map's with every output row shifted by the first map's output count.
__global__ void k_concat_rows(const int32_t* __restrict__ a_rows, int64_t a_slots, const int32_t* __restrict__ b_rows,
                              int64_t b_slots, int32_t shift, int32_t* __restrict__ rows) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < a_slots) {
    rows[i] = a_rows[i];
  } else if (i < a_slots + b_slots) {
    const int32_t r = b_rows[i - a_slots];
    rows[i] = r >= 0 ? r + shift : -1;
  }
}

// Pair counters of a concatenated map are the sums of its parts'; the build
// status is the first part's error, else the second's.
__global__ void k_concat_counters(const unsigned long long* a, const int* a_err, const unsigned long long* b,
                                  const int* b_err, unsigned long long* c, int* c_err) {
  if (threadIdx.x == 0) {
    c[0] = a[0] + b[0];
    c[1] = a[1] + b[1];
    *c_err = *a_err ? *a_err : *b_err;
  }
}

__global__ void k_iota(uint32_t* v, int64_t n) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) v[i] = static_cast<uint32_t>(i);
}

// Inserts every voxel's key; the same threads also fill the map with -1 and
// zero the row masks that the half-neighbourhood probe completes afterwards.
__global__ void k_hash_insert(const int4* __restrict__ coords, int64_t n, Slot* slots, uint32_t cap_mask, int* err,
                              int32_t* __restrict__ map, int64_t map_ints, uint32_t* __restrict__ row_mask,
                              int64_t n_out) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e = i; e < map_ints / 4; e += stride) reinterpret_cast<int4*>(map)[e] = make_int4(-1, -1, -1, -1);
  for (int64_t e = (map_ints / 4) * 4 + i; e < map_ints; e += stride) map[e] = -1;
  for (int64_t e = i; e < n_out; e += stride) row_mask[e] = 0u;
  if (i >= n) return;
  const int4 c = coords[i];
  if (!coord_ok(c)) {
    record_error(err, SC_ERANGE);
    return;
  }
  const unsigned long long key = pack16(c.x, c.y, c.z, c.w);
  uint32_t hpos = home_slot(c.x, c.y, c.z, c.w, cap_mask);
  for (uint32_t it = 0; it <= cap_mask; ++it) {
    const unsigned long long prev = atomicCAS(&slots[hpos].key, kEmptyKey, key);
    if (prev == kEmptyKey) {
      slots[hpos].val = static_cast<int>(i);
      return;
    }
    if (prev == key) {
      record_error(err, SC_EDUP_COORD);
      return;
    }
    hpos = rehash_slot(key, it + 1, cap_mask);
  }
  record_error(err, SC_ENOMEM);
}

__device__ __forceinline__ void write_rows_and_count(const int32_t* s_map, int64_t row0, int64_t n, int K,
                                                     int32_t* __restrict__ map, uint32_t m,
                                                     unsigned long long* counters) {
  __syncthreads();
  const int rows = static_cast<int>(min(static_cast<int64_t>(blockDim.x), n - row0));
  const int total = rows * K;
  for (int j = threadIdx.x; j < total; j += blockDim.x) map[row0 * K + j] = s_map[j];
  unsigned cnt = __popc(m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if ((threadIdx.x & 31) == 0 && cnt) atomicAdd(&counters[0], static_cast<unsigned long long>(cnt));
}

// Slow path of a probe whose home slot holds another key: follow the rehash
// sequence until the key or an empty slot is found.
__device__ __noinline__ int probe_chain(const ulonglong2* __restrict__ sl, unsigned long long q, uint32_t cap_mask) {
  for (uint32_t round = 1; round <= cap_mask; ++round) {
    const ulonglong2 s = __ldg(sl + rehash_slot(q, round, cap_mask));
    if (s.x == q) return static_cast<int>(static_cast<uint32_t>(s.y));
    if (s.x == kEmptyKey) return -1;
  }
  return -1;
}

// Half-neighbourhood probe, one thread per INPUT row a (all n rows): it looks
// up only the 13 offsets v = 0..12 (the mirror of offset v is 26 - v) and,
// when a's neighbour at v is row b,
//   * if a is an output row: map[a - out_lo][v] = b;
//   * if b is an output row: map[b - out_lo][26 - v] = a.
// Neighbourhood is symmetric (b is a's neighbour at v exactly when a is b's
// at 26 - v), so the two writes fill every entry of every output row with
// half the probes of a full lookup; entries no pair reaches keep the -1 the
// map was filled with, and each entry is written by exactly one thread.  Row
// masks collect both kinds of bits with atomicOr (zeroed first).  Home slots
// come from per-axis hash terms computed once; the 13 home-slot loads are
// issued together (out-of-range neighbours read a harmless slot and are
// discarded), and only a home slot holding another key takes the rehash slow
// path (rare at load <= 1/4).  Each warp stages the lower half and centre of
// its output rows in shared memory and writes them row by row.
__global__ void __launch_bounds__(256, 4) k_probe_hash(const int4* __restrict__ coords, int64_t n, int64_t out_lo,
                                                    int64_t out_hi, const Slot* __restrict__ slots, uint32_t cap_mask,
                                                    int dil_x, int dil_y, int dil_z, int32_t* __restrict__ map,
                                                    uint32_t* __restrict__ row_mask, unsigned long long* counters) {
  constexpr int kHalf = 14;  // offsets 0..12 and the centre
  __shared__ int32_t s_rows[8][32 * kHalf];
  const int lane = threadIdx.x & 31;
  int32_t* srow = s_rows[threadIdx.x >> 5] + lane * kHalf;
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const bool is_out = i >= out_lo && i < out_hi;
  uint32_t own = 0;
  unsigned cnt = 0;
  if (i < n) {
    const int4 c = coords[i];
    const bool cok = coord_ok(c);
    const unsigned long long base = pack16(c.x, c.y, c.z, c.w);
    const uint32_t hb = axis_term(c.x, kMulB);
    uint32_t hx[2], hy[3], hz[3], lx[2], ly[3], lz[3];
    bool vx[2], vy[3], vz[3];
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      const int x = c.y + (a - 1) * dil_x, y = c.z + (a - 1) * dil_y, z = c.w + (a - 1) * dil_z;
      if (a < 2) {
        vx[a] = cok && static_cast<unsigned>(x) <= 65535u;
        hx[a] = axis_term(x >> 2, kMulX);
        lx[a] = static_cast<uint32_t>(x & 3) << 4;
      }
      vy[a] = cok && static_cast<unsigned>(y) <= 65535u;
      vz[a] = cok && static_cast<unsigned>(z) <= 65535u;
      hy[a] = axis_term(y >> 2, kMulY);
      hz[a] = axis_term(z >> 2, kMulZ);
      ly[a] = static_cast<uint32_t>(y & 3) << 2;
      lz[a] = static_cast<uint32_t>(z & 3);
    }
    const ulonglong2* sl = reinterpret_cast<const ulonglong2*>(slots);
    ulonglong2 sv[13];
#pragma unroll
    for (int v = 0; v < 13; ++v) {
      const int a = v / 9, bb = (v / 3) % 3, cc = v % 3;
      const uint32_t pos = ((fin32(hb ^ hx[a] ^ hy[bb] ^ hz[cc]) << 6) | lx[a] | ly[bb] | lz[cc]) & cap_mask;
      sv[v] = __ldg(sl + pos);
    }
#pragma unroll
    for (int v = 0; v < 13; ++v) {
      const int a = v / 9, bb = (v / 3) % 3, cc = v % 3;
      const long long dq = (static_cast<long long>((a - 1) * dil_x) << 32) +
                           (static_cast<long long>((bb - 1) * dil_y) << 16) + static_cast<long long>((cc - 1) * dil_z);
      const unsigned long long q = base + static_cast<unsigned long long>(dq);
      int r = -1;
      if (vx[a] && vy[bb] && vz[cc]) {
        if (sv[v].x == q) r = static_cast<int>(static_cast<uint32_t>(sv[v].y));
        else if (sv[v].x != kEmptyKey) r = probe_chain(sl, q, cap_mask);
      }
      srow[v] = r;
      if (r >= 0) {
        if (is_out) {
          own |= 1u << v;
          ++cnt;
        }
        if (r >= out_lo && r < out_hi) {
          map[(static_cast<int64_t>(r) - out_lo) * 27 + (26 - v)] = static_cast<int32_t>(i);
          atomicOr(&row_mask[r - out_lo], 1u << (26 - v));
          ++cnt;
        }
      }
    }
    srow[13] = static_cast<int32_t>(i);
    if (is_out) {
      own |= 1u << 13;
      ++cnt;
      atomicOr(&row_mask[i - out_lo], own);
    }
  }
  __syncwarp();
  const int64_t first = i - lane;
  if (first < n) {
    const int32_t* src = s_rows[threadIdx.x >> 5];
    for (int e = lane; e < 32 * kHalf; e += 32) {
      const int64_t row = first + e / kHalf;
      if (row >= out_lo && row < out_hi && row < n) map[(row - out_lo) * 27 + e % kHalf] = src[e];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if ((threadIdx.x & 31) == 0 && cnt) atomicAdd(&counters[0], static_cast<unsigned long long>(cnt));
}

// ---------------------------------------------------------------- sort mode
struct Packing {
  int wx, wy, wz;     // bit widths of x, y, z fields
  int mx, my, mz;     // maxima (neighbours beyond them do not exist)
};

__device__ __forceinline__ unsigned long long pack_compact(int b, int x, int y, int z, const Packing& pk) {
  return (((static_cast<unsigned long long>(b) << pk.wx | static_cast<unsigned long long>(x)) << pk.wy |
           static_cast<unsigned long long>(y))
          << pk.wz) |
         static_cast<unsigned long long>(z);
}

__global__ void k_minmax(const int4* __restrict__ coords, int64_t n, int shift, int* maxes, int* err) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  int4 c = make_int4(0, 0, 0, 0);
  if (i < n) {
    c = coords[i];
    if (!coord_ok(c)) {
      record_error(err, SC_ERANGE);
      c = make_int4(0, 0, 0, 0);
    }
  }
  int mb = c.x, mx = c.y >> shift, my = c.z >> shift, mz = c.w >> shift;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    my = max(my, __shfl_xor_sync(0xffffffffu, my, o));
    mz = max(mz, __shfl_xor_sync(0xffffffffu, mz, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMax(&maxes[0], mb);
    atomicMax(&maxes[1], mx);
    atomicMax(&maxes[2], my);
    atomicMax(&maxes[3], mz);
  }
}

__global__ void k_pack_keys(const int4* __restrict__ coords, int64_t n, int shift, Packing pk,
                            unsigned long long* keys, uint32_t* vals) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  int4 c = coords[i];
  if (!coord_ok(c)) c = make_int4(0, 0, 0, 0);  // error already recorded by k_minmax
  keys[i] = pack_compact(c.x, c.y >> shift, c.z >> shift, c.w >> shift, pk);
  vals[i] = static_cast<uint32_t>(i);
}

__global__ void k_check_sorted_unique(const unsigned long long* __restrict__ skeys, int64_t n, int* err) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= 1 && i < n && skeys[i] == skeys[i - 1]) record_error(err, SC_EDUP_COORD);
}

__device__ __forceinline__ int sorted_find(const unsigned long long* __restrict__ skeys,
                                           const uint32_t* __restrict__ svals, int64_t n, unsigned long long q) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (__ldg(skeys + mid) < q) lo = mid + 1; else hi = mid;
  }
  return (lo < n && __ldg(skeys + lo) == q) ? static_cast<int>(__ldg(svals + lo)) : -1;
}

__global__ void __launch_bounds__(128) k_probe_sorted(const int4* __restrict__ coords, int64_t n, int64_t row_base,
                                                      const unsigned long long* __restrict__ skeys,
                                                      const uint32_t* __restrict__ svals, int64_t n_keys,
                                                      Packing pk, Dil dil,
                                                      int32_t* __restrict__ map, uint32_t* __restrict__ row_mask,
                                                      unsigned long long* counters) {
  __shared__ int32_t s_map[128 * 27];
  const int64_t row0 = blockIdx.x * 128ll;
  const int64_t i = row0 + threadIdx.x;
  uint32_t m = 0;
  if (i < n) {
    int4 c = coords[i];
    const bool cok = coord_ok(c);
#pragma unroll 1
    for (int v = 0; v < 27; ++v) {
      int dx, dy, dz;
      offset27(v, dil, dx, dy, dz);
      const int x = c.y + dx, y = c.z + dy, z = c.w + dz;
      int r = -1;
      if (v == 13) {
        r = static_cast<int>(row_base + i);
      } else if (cok && x >= 0 && y >= 0 && z >= 0 && x <= pk.mx && y <= pk.my && z <= pk.mz) {
        r = sorted_find(skeys, svals, n_keys, pack_compact(c.x, x, y, z, pk));
      }
      s_map[threadIdx.x * 27 + v] = r;
      m |= (r >= 0 ? 1u : 0u) << v;
    }
    row_mask[i] = m;
  }
  write_rows_and_count(s_map, row0, n, 27, map, m, counters);
}

// --------------------------------------------------------- down / up maps
// Scan helpers (3 kernels, no inter-block waits): parent id of every sorted entry.
constexpr int kScanBlock = 1024;

__global__ void k_heads_count(const unsigned long long* __restrict__ skeys, int64_t n, uint32_t* block_sums) {
  __shared__ uint32_t s[32];
  const int64_t i0 = blockIdx.x * static_cast<int64_t>(kScanBlock);
  uint32_t c = 0;
  for (int j = threadIdx.x; j < kScanBlock; j += blockDim.x) {
    const int64_t i = i0 + j;
    if (i < n && (i == 0 || skeys[i] != skeys[i - 1])) ++c;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += s[w];
    block_sums[blockIdx.x] = t;
  }
}

__global__ void k_scan_block_sums(uint32_t* block_sums, int64_t nb, uint32_t* total) {
  // single block of 1024 threads; exclusive scan in place, in chunks
  __shared__ uint32_t s[1024];
  uint32_t carry = 0;
  for (int64_t base = 0; base < nb; base += 1024) {
    const int64_t i = base + threadIdx.x;
    const uint32_t x = i < nb ? block_sums[i] : 0u;
    s[threadIdx.x] = x;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {
      const uint32_t y = threadIdx.x >= static_cast<unsigned>(o) ? s[threadIdx.x - o] : 0u;
      __syncthreads();
      s[threadIdx.x] += y;
      __syncthreads();
    }
    if (i < nb) block_sums[i] = carry + s[threadIdx.x] - x;
    const uint32_t chunk_total = s[1023];
    __syncthreads();
    carry += chunk_total;
  }
  if (threadIdx.x == 0) *total = carry;
}

__global__ void k_heads_assign(const unsigned long long* __restrict__ skeys, int64_t n,
                               const uint32_t* __restrict__ block_sums, uint32_t* __restrict__ pid) {
  // 1024 threads per block, one element each
  __shared__ uint32_t s[1024];
  const int64_t i = blockIdx.x * static_cast<int64_t>(kScanBlock) + threadIdx.x;
  const uint32_t f = (i < n && (i == 0 || skeys[i] != skeys[i - 1])) ? 1u : 0u;
  s[threadIdx.x] = f;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const uint32_t y = threadIdx.x >= static_cast<unsigned>(o) ? s[threadIdx.x - o] : 0u;
    __syncthreads();
    s[threadIdx.x] += y;
    __syncthreads();
  }
  if (i < n) pid[i] = block_sums[blockIdx.x] + s[threadIdx.x] - 1u;
}

__global__ void k_down_fill(const unsigned long long* __restrict__ skeys, const uint32_t* __restrict__ svals,
                            const uint32_t* __restrict__ pid, const int4* __restrict__ coords, int64_t n,
                            int32_t* dmap, int32_t* out_coords, int32_t* parent_code, int* err) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  const uint32_t c = svals[i];
  const uint32_t p = pid[i];
  const int4 cc = coords[c];
  const int slot = (cc.y & 1) * 4 + (cc.z & 1) * 2 + (cc.w & 1);
  const int prev = atomicExch(&dmap[static_cast<int64_t>(p) * 8 + slot], static_cast<int>(c));
  if (prev != -1) record_error(err, SC_EDUP_COORD);
  parent_code[c] = static_cast<int32_t>(p * 8u + static_cast<uint32_t>(slot));
  if (i == 0 || skeys[i] != skeys[i - 1]) {
    reinterpret_cast<int4*>(out_coords)[p] = make_int4(cc.x, cc.y >> 1, cc.z >> 1, cc.w >> 1);
  }
}

__global__ void k_row_masks(const int32_t* __restrict__ map, int64_t n, int K, uint32_t* row_mask,
                            unsigned long long* counters) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  uint32_t m = 0;
  if (i < n) {
    for (int v = 0; v < K; ++v) m |= (map[i * K + v] >= 0 ? 1u : 0u) << v;
    row_mask[i] = m;
  }
  unsigned cnt = __popc(m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if ((threadIdx.x & 31) == 0 && cnt) atomicAdd(&counters[0], static_cast<unsigned long long>(cnt));
}

__global__ void k_up_fill(const int32_t* __restrict__ parent_code, int64_t n, int32_t* umap, uint32_t* row_mask) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  const int32_t code = parent_code[i];
  const int slot = code & 7;
  umap[i * 8 + slot] = code >> 3;
  row_mask[i] = 1u << slot;
}

// ------------------------------------------------------------- tile layout
__global__ void __launch_bounds__(128) k_build_tiles(const int32_t* __restrict__ map, int K,
                                                     const uint32_t* __restrict__ perm, int64_t n_out,
                                                     const uint32_t* __restrict__ row_mask, int32_t* gidx,
                                                     int32_t* tile_rows, uint32_t* tile_mask,
                                                     unsigned long long* counters) {
  __shared__ uint32_t s_or[4];
  const int64_t t = blockIdx.x;
  const int i = threadIdx.x;
  const int64_t s = t * kTileRows + i;
  const int r = s < n_out ? static_cast<int>(perm[s]) : -1;
  tile_rows[s] = r;
  uint32_t m = r >= 0 ? row_mask[r] : 0u;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m |= __shfl_xor_sync(0xffffffffu, m, o);
  if ((i & 31) == 0) s_or[i >> 5] = m;
  for (int v = 0; v < K; ++v) {
    gidx[(t * K + v) * kTileRows + i] = r >= 0 ? __ldg(map + static_cast<int64_t>(r) * K + v) : -1;
  }
  __syncthreads();
  if (i == 0) {
    const uint32_t tm = s_or[0] | s_or[1] | s_or[2] | s_or[3];
    tile_mask[t] = tm;
    atomicAdd(&counters[1], static_cast<unsigned long long>(kTileRows) * __popc(tm));
  }
}

__global__ void k_export(const int32_t* __restrict__ gidx, const int32_t* __restrict__ tile_rows, int64_t num_tiles,
                         int K, int32_t* __restrict__ map_out) {
  const int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (e >= num_tiles * K * kTileRows) return;
  const int i = static_cast<int>(e % kTileRows);
  const int64_t tv = e / kTileRows;
  const int64_t t = tv / K;
  const int v = static_cast<int>(tv % K);
  const int r = tile_rows[t * kTileRows + i];
  if (r >= 0) map_out[static_cast<int64_t>(r) * K + v] = gidx[e];
}

inline unsigned blocks_for(int64_t n, int threads) { return static_cast<unsigned>((n + threads - 1) / threads); }

int bit_width(int v) {
  int w = 0;
  while (w < 31 && (v >> w) != 0) ++w;
  return w;
}

// RAII list of stream-ordered temporaries.
struct Temps {
  Handle* h;
  std::vector<void*> ptrs;
  explicit Temps(Handle* hh) : h(hh) {}
  ~Temps() {
    for (void* p : ptrs) dev_free(h, p);
  }
  template <typename T>
  cudaError_t get(T** p, size_t bytes) {
    void* q = nullptr;
    cudaError_t e = dev_alloc(h, &q, bytes ? bytes : 16);
    if (e == cudaSuccess) ptrs.push_back(q);
    *p = static_cast<T*>(q);
    return e;
  }
};

#define SC_TRY_CUDA(expr, what)                 \
  do {                                          \
    cudaError_t _e = (expr);                    \
    if (_e != cudaSuccess) return cuda_error(h, _e, what); \
  } while (0)

// Allocates the persistent parts of a map (owned by the KMap).
sc_status alloc_kmap(Handle* h, KMap* km) {
  km->num_tiles = (km->n_out + kTileRows - 1) / kTileRows;
  const int64_t slots = std::max<int64_t>(km->num_tiles, 1) * kTileRows;
  SC_TRY_CUDA(dev_alloc(h, reinterpret_cast<void**>(&km->gidx), sizeof(int32_t) * slots * km->K), "alloc gidx");
  SC_TRY_CUDA(dev_alloc(h, reinterpret_cast<void**>(&km->tile_rows), sizeof(int32_t) * slots), "alloc tile_rows");
  SC_TRY_CUDA(dev_alloc(h, reinterpret_cast<void**>(&km->tile_mask),
                        sizeof(uint32_t) * std::max<int64_t>(km->num_tiles, 1)),
              "alloc tile_mask");
  return SC_OK;
}

// Sort key of a row for tile formation: the 26 non-centre bits of its 3x3x3
// mask reordered as face neighbours (low bits), edge neighbours, then corner
// neighbours (most significant), so rows that share corner/edge patterns sort
// together.  On the 256^3 shell workload this ordering raises the useful
// fraction of tile work from 0.72 (mask value order) to 0.75.  2x2x2 maps use
// the mask itself.  Sorting on 16 instead of 24 key bits (two passes instead
// of three) would drop it to 0.72 (0.84 instead of 0.93 on the 1024^3 shell).
__device__ __forceinline__ uint32_t tile_sort_key(uint32_t m, int K) {
  if (K != 27) return m;
  uint32_t k = 0;
  int pos = 0;
#pragma unroll
  for (int cls = 1; cls <= 3; ++cls) {
#pragma unroll
    for (int v = 0; v < 27; ++v) {
      const int ad = (v / 9 == 1 ? 0 : 1) + ((v / 3) % 3 == 1 ? 0 : 1) + (v % 3 == 1 ? 0 : 1);
      if (ad == cls) {
        k |= ((m >> v) & 1u) << pos;
        ++pos;
      }
    }
  }
  return k;
}

// Writes every row's sort key and the identity permutation, and adds the
// key digits of every radix pass (8 bits from begin_bit each) into the
// sort's histogram: the sort then starts with its first scatter pass.
constexpr int kKeyHistPasses = 4;
__global__ void __launch_bounds__(256) k_sort_keys(const uint32_t* __restrict__ row_mask, int64_t n, int K,
                                                   int begin_bit, int passes, uint32_t* __restrict__ keys,
                                                   uint32_t* __restrict__ perm, uint32_t* __restrict__ ghist) {
  __shared__ uint32_t h[kKeyHistPasses][kRadixBins];
  for (int e = threadIdx.x; e < kKeyHistPasses * kRadixBins; e += blockDim.x) (&h[0][0])[e] = 0;
  __syncthreads();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t k = tile_sort_key(row_mask[i], K);
    keys[i] = k;
    perm[i] = static_cast<uint32_t>(i);
    for (int p = 0; p < passes; ++p) atomicAdd(&h[p][(k >> (begin_bit + 8 * p)) & 0xFFu], 1u);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < passes * kRadixBins; e += blockDim.x) {
    const uint32_t c = (&h[0][0])[e];
    if (c) atomicAdd(&ghist[e], c);
  }
}

// Work order of tile groups for the conv's scheduler: groups of `tpi`
// consecutive tiles bucketed by the number of offsets they run (descending),
// a counting sort in two passes (bucket sizes, then placement).  The order
// within a bucket depends on atomic timing; conv results do not, since every
// output row sums its offsets in the same order whichever CTA computes it.
// Groups holding a tile at or past `split` (the second part of a concatenated
// map) form a second class of buckets placed after the first.
constexpr int kWorkBuckets = 66;  // (late class) x (offsets per group: 0..32)

__device__ __forceinline__ int group_bucket(const uint32_t* tile_mask, int64_t g, int64_t num_tiles, int tpi,
                                            int64_t split) {
  uint32_t m = 0;
  for (int i = 0; i < tpi; ++i)
    if (g * tpi + i < num_tiles) m |= tile_mask[g * tpi + i];
  const int64_t end = (g + 1) * tpi < num_tiles ? (g + 1) * tpi : num_tiles;
  return 32 - __popc(m) + (end > split ? 33 : 0);  // more offsets first, late class last
}

// The work orders of groups of one, two and four tiles in one single-CTA
// launch: bucket counts in shared memory, an exclusive scan turns them into
// placement cursors, and a second pass places every group.  An order is
// written only where its pointer is non-null.
constexpr int kOrderThreads = 1024;
constexpr int kOrders = 3;  // tiles per group 1 << k

__global__ void __launch_bounds__(kOrderThreads) k_group_orders(const uint32_t* __restrict__ tile_mask,
                                                                int64_t num_tiles, int64_t split, int32_t* order1,
                                                                int32_t* order2, int32_t* order4) {
  __shared__ uint32_t cur[kOrders][kWorkBuckets];
  int32_t* const orders[kOrders] = {order1, order2, order4};
  for (int b = threadIdx.x; b < kOrders * kWorkBuckets; b += blockDim.x) cur[b / kWorkBuckets][b % kWorkBuckets] = 0;
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kOrders; ++k) {
    if (!orders[k]) continue;
    const int tpi = 1 << k;
    const int64_t groups = (num_tiles + tpi - 1) / tpi;
    for (int64_t g = threadIdx.x; g < groups; g += blockDim.x)
      atomicAdd(&cur[k][group_bucket(tile_mask, g, num_tiles, tpi, split)], 1u);
  }
  __syncthreads();
  if (threadIdx.x < kOrders) {
    uint32_t acc = 0;
    for (int b = 0; b < kWorkBuckets; ++b) {
      const uint32_t c = cur[threadIdx.x][b];
      cur[threadIdx.x][b] = acc;
      acc += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kOrders; ++k) {
    int32_t* order = orders[k];
    if (!order) continue;
    const int tpi = 1 << k;
    const int64_t groups = (num_tiles + tpi - 1) / tpi;
    for (int64_t g = threadIdx.x; g < groups; g += blockDim.x)
      order[atomicAdd(&cur[k][group_bucket(tile_mask, g, num_tiles, tpi, split)], 1u)] = static_cast<int32_t>(g);
  }
}

// Orders output rows by neighbour mask and writes gidx / tile_rows / tile_mask.

// Halo lists of output-order tiles (one CTA per tile).  The 27 x 128 gathered
// rows are deduplicated in a shared-memory hash set; the set is compacted into
// the tile's halo list (order = slot order) and every gathered row is replaced
// by its position in the list.  A tile's halo count above kHaloCap (or a full
// set, which can only happen past the cap) marks it for direct gathers.
constexpr int kHaloSlots = 1024;
constexpr int kHaloThreads = 256;

__device__ __forceinline__ uint32_t halo_hash(int r) {
  return (static_cast<uint32_t>(r) * 0x9E3779B1u) >> (32 - 10);
}

__global__ void __launch_bounds__(kHaloThreads) k_build_halo(const int32_t* __restrict__ map, int64_t n_out,
                                                             int32_t* __restrict__ halo_rows,
                                                             int32_t* __restrict__ halo_n, uint16_t* __restrict__ lidx,
                                                             unsigned long long* hmax) {
  static_assert(kHaloSlots == 1 << 10, "halo_hash assumes 1024 slots");
  __shared__ int tab[kHaloSlots];   // row or -1
  __shared__ int pos[kHaloSlots];   // position in the halo list
  __shared__ int s_warp[kHaloThreads / 32];
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  for (int e = tid; e < kHaloSlots; e += kHaloThreads) tab[e] = -1;
  __syncthreads();
  const int64_t base = t * kTileRows * 27;
  const int64_t lim = (n_out - t * kTileRows) * 27;  // valid map entries of this tile
  for (int e = tid; e < kTileRows * 27; e += kHaloThreads) {
    const int r = e < lim ? map[base + e] : -1;
    if (r < 0) continue;
    uint32_t hh = halo_hash(r);
    for (int probe = 0; probe < kHaloSlots; ++probe) {
      const int old = atomicCAS(&tab[hh], -1, r);
      if (old == -1 || old == r) break;
      hh = (hh + 1) & (kHaloSlots - 1);
    }
  }
  __syncthreads();
  constexpr int kPer = kHaloSlots / kHaloThreads;
  int cnt = 0;
#pragma unroll
  for (int k = 0; k < kPer; ++k) cnt += tab[tid * kPer + k] >= 0 ? 1 : 0;
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if ((tid & 31) >= o) incl += y;
  }
  if ((tid & 31) == 31) s_warp[tid >> 5] = incl;
  __syncthreads();
  int wbase = 0, total = 0;
  for (int w = 0; w < kHaloThreads / 32; ++w) {
    if (w < (tid >> 5)) wbase += s_warp[w];
    total += s_warp[w];
  }
  // A full table may have dropped rows; it can only fill past the cap.
  if (total >= kHaloSlots) total = kHaloSlots + 1;
  int p = wbase + incl - cnt;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int sidx = tid * kPer + k;
    const int r = tab[sidx];
    if (r >= 0) {
      pos[sidx] = p;
      if (p < kHaloCap) halo_rows[t * kHaloCap + p] = r;
      ++p;
    }
  }
  // pad to a multiple of 4 rows (the conv gathers 4 rows per TMA instruction;
  // row -1 reads zeros)
  const int padded = min((total + 3) & ~3, kHaloCap);
  for (int q = total + tid; q < padded; q += kHaloThreads) halo_rows[t * kHaloCap + q] = -1;
  if (tid == 0) {
    halo_n[t] = total;
    atomicMax(hmax, static_cast<unsigned long long>(total));
  }
  if (total > kHaloCap) return;  // direct gathers: no positions needed
  __syncthreads();
  for (int e = tid; e < kTileRows * 27; e += kHaloThreads) {
    const int v = e / kTileRows, i = e - v * kTileRows;
    const int64_t ei = static_cast<int64_t>(i) * 27 + v;
    const int r = ei < lim ? map[base + ei] : -1;
    uint16_t l = 0xFFFFu;
    if (r >= 0) {
      uint32_t hh = halo_hash(r);
      for (int probe = 0; probe < kHaloSlots && tab[hh] != r; ++probe) hh = (hh + 1) & (kHaloSlots - 1);
      l = static_cast<uint16_t>(pos[hh]);
    }
    lidx[(t * 27 + v) * kTileRows + i] = l;
  }
}

sc_status build_halo(Handle* h, KMap* km, const int32_t* map) {
  const int64_t T = km->num_tiles;
  SC_TRY_CUDA(dev_alloc(h, reinterpret_cast<void**>(&km->halo_rows), sizeof(int32_t) * T * kHaloCap), "alloc halo");
  SC_TRY_CUDA(dev_alloc(h, reinterpret_cast<void**>(&km->halo_n), sizeof(int32_t) * T), "alloc halo");
  SC_TRY_CUDA(dev_alloc(h, reinterpret_cast<void**>(&km->lidx), sizeof(uint16_t) * T * 27 * kTileRows), "alloc halo");
  ++h->launches;
  k_build_halo<<<static_cast<unsigned>(T), kHaloThreads, 0, h->stream>>>(map, km->n_out, km->halo_rows, km->halo_n,
                                                                         km->lidx, km->counters + 2);
  SC_TRY_CUDA(cudaGetLastError(), "halo launch");
  return SC_OK;
}

// Work orders of the conv's scheduler (1, 2 and 4 tiles per item), built with
// the map on its stream so
// that whatever is ordered after the build (any stream, any handle) sees
// them.  A conv uses the order of its tiles-per-item count only when it runs
// fewer than kWorkOrderMaxItemsPerCta items per CTA, and it runs at least one
// item per group, so orders of kWorkOrderMaxItemsPerCta * num_sms groups or
// more are never read and are not built.
sc_status build_group_orders(Handle* h, KMap* km) {
  if (km->num_tiles == 0) return SC_OK;
  const int64_t split = km->split_tile >= 0 ? km->split_tile : km->num_tiles;
  bool any = false;
  for (int t = 0; t < kOrders; ++t) {
    const int64_t tpi = int64_t{1} << t;
    const int64_t groups = (km->num_tiles + tpi - 1) / tpi;
    if (groups < kWorkOrderMaxItemsPerCta * h->num_sms) {
      SC_TRY_CUDA(dev_alloc(h, reinterpret_cast<void**>(&km->group_order[t]), sizeof(int32_t) * groups),
                  "alloc group order");
      any = true;
    }
  }
  if (!any) return SC_OK;
  ++h->launches;
  k_group_orders<<<1, kOrderThreads, 0, h->stream>>>(km->tile_mask, km->num_tiles, split, km->group_order[0],
                                                      km->group_order[1], km->group_order[2]);
  SC_TRY_CUDA(cudaGetLastError(), "group order launch");
  return SC_OK;
}

sc_status finish_tiles(Handle* h, KMap* km, const int32_t* map, uint32_t* row_mask, uint32_t flags, Temps& tmp) {
  const int64_t n = km->n_out;
  if (n == 0) return SC_OK;
  uint32_t *perm, *perm_alt, *mask_alt, *mask_copy;
  SC_TRY_CUDA(tmp.get(&perm, sizeof(uint32_t) * n), "alloc perm");
  const uint32_t* order = perm;
  if (flags & SC_BUILD_NO_TILE_SORT) {
    ++h->launches;
    k_iota<<<blocks_for(n, 256), 256, 0, h->stream>>>(perm, n);
  } else {
    SC_TRY_CUDA(tmp.get(&perm_alt, sizeof(uint32_t) * n), "alloc perm");
    SC_TRY_CUDA(tmp.get(&mask_alt, sizeof(uint32_t) * n), "alloc masks");
    SC_TRY_CUDA(tmp.get(&mask_copy, sizeof(uint32_t) * n), "alloc masks");
    // 3x3x3 maps sort on the top 24 of the 26 key bits (three 8-bit passes
    // instead of four): on the 256^3 workload the useful fraction of tile rows
    // goes from 0.754 to 0.752 while one sort pass (~13 us) disappears.
    const int begin_bit = km->K == 27 ? 2 : 0;
    const int end_bit = km->K == 27 ? 26 : km->K;
    const int passes = (end_bit - begin_bit + 7) / 8;
    const size_t tb = radix_sort_temp_bytes(n, 4, passes);
    void* temp;
    SC_TRY_CUDA(tmp.get(&temp, tb), "alloc sort temp");
    SC_TRY_CUDA(cudaMemsetAsync(temp, 0, tb, h->stream), "clear sort temp");
    ++h->launches;
    const unsigned kgrid = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 4 * h->num_sms));
    k_sort_keys<<<kgrid, 256, 0, h->stream>>>(row_mask, n, km->K, begin_bit, passes, mask_copy, perm,
                                              static_cast<uint32_t*>(temp));
    bool in_alt = false;
    sc_status st = radix_sort_pairs_u32(h, mask_copy, perm, mask_alt, perm_alt, n, begin_bit, end_bit, temp, tb,
                                        km->err, &in_alt, /*hist_ready=*/true);
    if (st != SC_OK) return st;
    order = in_alt ? perm_alt : perm;
  }
  ++h->launches;
  k_build_tiles<<<static_cast<unsigned>(km->num_tiles), kTileRows, 0, h->stream>>>(
      map, km->K, order, n, row_mask, km->gidx, km->tile_rows, km->tile_mask, km->counters);
  SC_TRY_CUDA(cudaGetLastError(), "tile build launch");
  return build_group_orders(h, km);
}


sc_status new_kmap(Handle* h, int kind, int K, int64_t n_in, int64_t n_out, KMap** out) {
  KMap* km = new (std::nothrow) KMap();
  if (!km) return set_error(h, SC_ENOMEM, "host allocation failed");
  km->kind = kind;
  km->K = K;
  km->n_in = n_in;
  km->n_out = n_out;
  cudaError_t e = dev_alloc(h, reinterpret_cast<void**>(&km->counters), 64);
  if (e == cudaSuccess) e = cudaMemsetAsync(km->counters, 0, 64, h->stream);
  if (e != cudaSuccess) {
    free_kmap(h, km);
    return cuda_error(h, e, "alloc kmap counters");
  }
  km->err = reinterpret_cast<int*>(km->counters + 4);
  *out = km;
  return SC_OK;
}

// Reads the device maxima of (b, x>>shift, y>>shift, z>>shift); synchronises.
sc_status read_maxima(Handle* h, const int32_t* coords, int64_t n, int shift, int* err, Temps& tmp, int hmax[4]) {
  int* dmax;
  SC_TRY_CUDA(tmp.get(&dmax, 16), "alloc maxima");
  SC_TRY_CUDA(cudaMemsetAsync(dmax, 0, 16, h->stream), "memset maxima");
  ++h->launches;
  k_minmax<<<blocks_for(n, 256), 256, 0, h->stream>>>(reinterpret_cast<const int4*>(coords), n, shift, dmax, err);
  int herr = 0;
  SC_TRY_CUDA(cudaMemcpyAsync(hmax, dmax, 16, cudaMemcpyDeviceToHost, h->stream), "copy maxima");
  SC_TRY_CUDA(cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, h->stream), "copy err");
  SC_TRY_CUDA(cudaStreamSynchronize(h->stream), "sync maxima");
  if (herr == SC_ERANGE) return set_error(h, SC_ERANGE, "coordinate out of range (b in [0, 32767], x/y/z in [0, 65535])");
  return SC_OK;
}

}  // namespace

sc_status build_subm(Handle* h, const int32_t* coords, int64_t n, int64_t out_begin, int64_t n_out, Dil dilation,
                     uint32_t flags, KMap** out) {
  // Neighbours are looked up among all n input rows; output j is input row
  // out_begin + j, for j in [0, n_out).
  KMap* km = nullptr;
  sc_status st = new_kmap(h, SC_KMAP_SUBM, 27, n, n_out, &km);
  if (st != SC_OK) return st;
  Temps tmp(h);
  st = alloc_kmap(h, km);
  if (st != SC_OK || n == 0 || n_out == 0) {
    if (st != SC_OK) free_kmap(h, km); else *out = km;
    return st;
  }
  int32_t* map;
  uint32_t* row_mask;
  cudaError_t e = tmp.get(&map, sizeof(int32_t) * n_out * 27);
  if (e == cudaSuccess) e = tmp.get(&row_mask, sizeof(uint32_t) * n_out);
  if (e != cudaSuccess) {
    free_kmap(h, km);
    return cuda_error(h, e, "alloc map");
  }
  const int4* c4 = reinterpret_cast<const int4*>(coords);
  if (h->map_mode == SC_MAP_SORT) {
    int hmax[4];
    st = read_maxima(h, coords, n, 0, km->err, tmp, hmax);
    if (st != SC_OK) {
      free_kmap(h, km);
      return st;
    }
    Packing pk{bit_width(hmax[1]), bit_width(hmax[2]), bit_width(hmax[3]), hmax[1], hmax[2], hmax[3]};
    const int bits = bit_width(hmax[0]) + pk.wx + pk.wy + pk.wz;
    unsigned long long *keys, *keys_alt;
    uint32_t *vals, *vals_alt;
    void* temp;
    const int passes = std::max(1, (bits + 7) / 8);
    const size_t tb = radix_sort_temp_bytes(n, 8, passes);
    e = tmp.get(&keys, 8 * n);
    if (e == cudaSuccess) e = tmp.get(&keys_alt, 8 * n);
    if (e == cudaSuccess) e = tmp.get(&vals, 4 * n);
    if (e == cudaSuccess) e = tmp.get(&vals_alt, 4 * n);
    if (e == cudaSuccess) e = tmp.get(&temp, tb);
    if (e != cudaSuccess) {
      free_kmap(h, km);
      return cuda_error(h, e, "alloc sort buffers");
    }
    ++h->launches;
    k_pack_keys<<<blocks_for(n, 256), 256, 0, h->stream>>>(c4, n, 0, pk, keys, vals);
    bool in_alt = false;
    st = radix_sort_pairs_u64(h, reinterpret_cast<uint64_t*>(keys), vals, reinterpret_cast<uint64_t*>(keys_alt),
                              vals_alt, n, 0, std::max(bits, 1), temp, tb, km->err, &in_alt);
    if (st != SC_OK) {
      free_kmap(h, km);
      return st;
    }
    const unsigned long long* sk = in_alt ? keys_alt : keys;
    const uint32_t* sv = in_alt ? vals_alt : vals;
    ++h->launches;
    k_check_sorted_unique<<<blocks_for(n, 256), 256, 0, h->stream>>>(sk, n, km->err);
    ++h->launches;
    k_probe_sorted<<<blocks_for(n_out, 128), 128, 0, h->stream>>>(c4 + out_begin, n_out, out_begin, sk, sv, n, pk,
                                                               dilation, map, row_mask, km->counters);
  } else {
    uint32_t cap = 4096;
    while (cap < 4 * n) cap <<= 1;
    Slot* slots;
    e = tmp.get(&slots, sizeof(Slot) * cap);
    if (e == cudaSuccess) e = cudaMemsetAsync(slots, 0xFF, sizeof(Slot) * cap, h->stream);
    if (e != cudaSuccess) {
      free_kmap(h, km);
      return cuda_error(h, e, "alloc hash table");
    }
    // the half-neighbourhood probe fills the rest of every map row by mirror
    // writes and ORs mask bits in: the insert sets the map to -1 and the
    // masks to 0 first
    ++h->launches;
    k_hash_insert<<<blocks_for(n, 256), 256, 0, h->stream>>>(c4, n, slots, cap - 1, km->err, map, n_out * 27,
                                                              row_mask, n_out);
    ++h->launches;
    k_probe_hash<<<blocks_for(n, 256), 256, 0, h->stream>>>(c4, n, out_begin, out_begin + n_out, slots, cap - 1,
                                                         dilation.x, dilation.y, dilation.z, map, row_mask,
                                                         km->counters);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    free_kmap(h, km);
    return cuda_error(h, e, "map build launch");
  }
  const bool halo = (flags & SC_BUILD_HALO) != 0;
  st = finish_tiles(h, km, map, row_mask, halo ? (flags | SC_BUILD_NO_TILE_SORT) : flags, tmp);
  if (st == SC_OK && halo) st = build_halo(h, km, map);
  if (st != SC_OK) {
    free_kmap(h, km);
    return st;
  }
  *out = km;
  return SC_OK;
}

sc_status build_down2(Handle* h, const int32_t* coords, int64_t n, uint32_t flags, KMap** out) {
  KMap* km = nullptr;
  sc_status st = new_kmap(h, SC_KMAP_DOWN2, 8, n, 0, &km);
  if (st != SC_OK) return st;
  Temps tmp(h);
  if (n == 0) {
    st = alloc_kmap(h, km);
    if (st != SC_OK) free_kmap(h, km); else *out = km;
    return st;
  }
  int hmax[4];
  st = read_maxima(h, coords, n, 1, km->err, tmp, hmax);
  if (st != SC_OK) {
    free_kmap(h, km);
    return st;
  }
  Packing pk{bit_width(hmax[1]), bit_width(hmax[2]), bit_width(hmax[3]), hmax[1], hmax[2], hmax[3]};
  const int bits = std::max(1, bit_width(hmax[0]) + pk.wx + pk.wy + pk.wz);
  const int passes = (bits + 7) / 8;
  const size_t tb = radix_sort_temp_bytes(n, 8, passes);
  unsigned long long *keys, *keys_alt;
  uint32_t *vals, *vals_alt, *pid, *bsums, *dtotal;
  void* temp;
  const int64_t nb = (n + kScanBlock - 1) / kScanBlock;
  cudaError_t e = tmp.get(&keys, 8 * n);
  if (e == cudaSuccess) e = tmp.get(&keys_alt, 8 * n);
  if (e == cudaSuccess) e = tmp.get(&vals, 4 * n);
  if (e == cudaSuccess) e = tmp.get(&vals_alt, 4 * n);
  if (e == cudaSuccess) e = tmp.get(&temp, tb);
  if (e == cudaSuccess) e = tmp.get(&pid, 4 * n);
  if (e == cudaSuccess) e = tmp.get(&bsums, 4 * nb);
  if (e == cudaSuccess) e = tmp.get(&dtotal, 16);
  if (e == cudaSuccess) e = dev_alloc(h, reinterpret_cast<void**>(&km->parent_of), 4 * n);
  if (e != cudaSuccess) {
    free_kmap(h, km);
    return cuda_error(h, e, "alloc down buffers");
  }
  const int4* c4 = reinterpret_cast<const int4*>(coords);
  ++h->launches;
  k_pack_keys<<<blocks_for(n, 256), 256, 0, h->stream>>>(c4, n, 1, pk, keys, vals);
  bool in_alt = false;
  st = radix_sort_pairs_u64(h, reinterpret_cast<uint64_t*>(keys), vals, reinterpret_cast<uint64_t*>(keys_alt),
                            vals_alt, n, 0, bits, temp, tb, km->err, &in_alt);
  if (st != SC_OK) {
    free_kmap(h, km);
    return st;
  }
  const unsigned long long* sk = in_alt ? keys_alt : keys;
  const uint32_t* sv = in_alt ? vals_alt : vals;
  ++h->launches;
  k_heads_count<<<static_cast<unsigned>(nb), 256, 0, h->stream>>>(sk, n, bsums);
  ++h->launches;
  k_scan_block_sums<<<1, 1024, 0, h->stream>>>(bsums, nb, dtotal);
  ++h->launches;
  k_heads_assign<<<static_cast<unsigned>(nb), 1024, 0, h->stream>>>(sk, n, bsums, pid);
  uint32_t np = 0;
  e = cudaMemcpyAsync(&np, dtotal, 4, cudaMemcpyDeviceToHost, h->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) {
    free_kmap(h, km);
    return cuda_error(h, e, "down-sample parent count");
  }
  km->n_out = np;
  st = alloc_kmap(h, km);
  if (st != SC_OK) {
    free_kmap(h, km);
    return st;
  }
  int32_t* dmap;
  uint32_t* row_mask;
  e = tmp.get(&dmap, sizeof(int32_t) * 8 * np);
  if (e == cudaSuccess) e = tmp.get(&row_mask, sizeof(uint32_t) * np);
  if (e == cudaSuccess) e = dev_alloc(h, reinterpret_cast<void**>(&km->out_coords), sizeof(int32_t) * 4 * np);
  if (e == cudaSuccess) e = cudaMemsetAsync(dmap, 0xFF, sizeof(int32_t) * 8 * np, h->stream);
  if (e != cudaSuccess) {
    free_kmap(h, km);
    return cuda_error(h, e, "alloc down map");
  }
  ++h->launches;
  k_down_fill<<<blocks_for(n, 256), 256, 0, h->stream>>>(sk, sv, pid, c4, n, dmap, km->out_coords, km->parent_of,
                                                          km->err);
  ++h->launches;
  k_row_masks<<<blocks_for(np, 256), 256, 0, h->stream>>>(dmap, np, 8, row_mask, km->counters);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    free_kmap(h, km);
    return cuda_error(h, e, "down map launch");
  }
  st = finish_tiles(h, km, dmap, row_mask, flags, tmp);
  if (st != SC_OK) {
    free_kmap(h, km);
    return st;
  }
  *out = km;
  return SC_OK;
}

sc_status build_up2(Handle* h, const KMap* down, uint32_t flags, KMap** out) {
  if (!down || down->kind != SC_KMAP_DOWN2) return set_error(h, SC_EINVAL, "up2 needs a down2 map");
  KMap* km = nullptr;
  sc_status st = new_kmap(h, SC_KMAP_UP2, 8, down->n_out, down->n_in, &km);
  if (st != SC_OK) return st;
  Temps tmp(h);
  st = alloc_kmap(h, km);
  if (st != SC_OK || km->n_out == 0) {
    if (st != SC_OK) free_kmap(h, km); else *out = km;
    return st;
  }
  const int64_t n = km->n_out;
  int32_t* umap;
  uint32_t* row_mask;
  cudaError_t e = tmp.get(&umap, sizeof(int32_t) * 8 * n);
  if (e == cudaSuccess) e = tmp.get(&row_mask, sizeof(uint32_t) * n);
  if (e == cudaSuccess) e = cudaMemsetAsync(umap, 0xFF, sizeof(int32_t) * 8 * n, h->stream);
  if (e != cudaSuccess) {
    free_kmap(h, km);
    return cuda_error(h, e, "alloc up map");
  }
  ++h->launches;
  k_up_fill<<<blocks_for(n, 256), 256, 0, h->stream>>>(down->parent_of, n, umap, row_mask);
  ++h->launches;
  k_row_masks<<<blocks_for(n, 256), 256, 0, h->stream>>>(umap, n, 8, row_mask, km->counters);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    free_kmap(h, km);
    return cuda_error(h, e, "up map launch");
  }
  st = finish_tiles(h, km, umap, row_mask, flags, tmp);
  if (st != SC_OK) {
    free_kmap(h, km);
    return st;
  }
  *out = km;
  return SC_OK;
}

sc_status export_map(Handle* h, const KMap* km, int32_t* map_out) {
  const int64_t n = km->n_out;
  if (n == 0) return SC_OK;
  cudaError_t e = cudaMemsetAsync(map_out, 0xFF, sizeof(int32_t) * n * km->K, h->stream);
  if (e != cudaSuccess) return cuda_error(h, e, "export memset");
  const int64_t tot = km->num_tiles * km->K * kTileRows;
  ++h->launches;
  k_export<<<blocks_for(tot, 256), 256, 0, h->stream>>>(km->gidx, km->tile_rows, km->num_tiles, km->K, map_out);
  e = cudaGetLastError();
  return e == cudaSuccess ? SC_OK : cuda_error(h, e, "export launch");
}

void free_kmap(Handle* h, KMap* km) {
  if (!km) return;
  dev_free(h, km->gidx);
  dev_free(h, km->tile_rows);
  dev_free(h, km->tile_mask);
  dev_free(h, km->halo_rows);
  dev_free(h, km->halo_n);
  dev_free(h, km->lidx);
  for (int32_t* o : km->group_order) dev_free(h, o);
  dev_free(h, km->out_coords);
  dev_free(h, km->parent_of);
  dev_free(h, km->counters);
  delete km;
}

sc_status concat_maps(Handle* h, const KMap* a, const KMap* b, KMap** out) {
  if (a->kind != SC_KMAP_SUBM || b->kind != SC_KMAP_SUBM || a->K != b->K || a->n_in != b->n_in)
    return set_error(h, SC_EINVAL, "concat: both maps must be submanifold maps over the same input rows");
  if (a->n_out + b->n_out >= (1ll << 31)) return set_error(h, SC_EINVAL, "concat: too many output rows");
  KMap* km = nullptr;
  sc_status st = new_kmap(h, SC_KMAP_SUBM, a->K, a->n_in, a->n_out + b->n_out, &km);
  if (st != SC_OK) return st;
  km->num_tiles = a->num_tiles + b->num_tiles;
  km->split_tile = a->num_tiles;
  const int64_t T = km->num_tiles, slots = std::max<int64_t>(T, 1) * kTileRows;
  cudaError_t e = dev_alloc(h, reinterpret_cast<void**>(&km->gidx), sizeof(int32_t) * slots * km->K);
  if (e == cudaSuccess) e = dev_alloc(h, reinterpret_cast<void**>(&km->tile_rows), sizeof(int32_t) * slots);
  if (e == cudaSuccess)
    e = dev_alloc(h, reinterpret_cast<void**>(&km->tile_mask), sizeof(uint32_t) * std::max<int64_t>(T, 1));
  const size_t ga = sizeof(int32_t) * a->num_tiles * a->K * kTileRows;
  const size_t gb = sizeof(int32_t) * b->num_tiles * b->K * kTileRows;
  if (e == cudaSuccess && ga) e = cudaMemcpyAsync(km->gidx, a->gidx, ga, cudaMemcpyDeviceToDevice, h->stream);
  if (e == cudaSuccess && gb)
    e = cudaMemcpyAsync(reinterpret_cast<uint8_t*>(km->gidx) + ga, b->gidx, gb, cudaMemcpyDeviceToDevice, h->stream);
  if (e == cudaSuccess && a->num_tiles)
    e = cudaMemcpyAsync(km->tile_mask, a->tile_mask, sizeof(uint32_t) * a->num_tiles, cudaMemcpyDeviceToDevice,
                        h->stream);
  if (e == cudaSuccess && b->num_tiles)
    e = cudaMemcpyAsync(km->tile_mask + a->num_tiles, b->tile_mask, sizeof(uint32_t) * b->num_tiles,
                        cudaMemcpyDeviceToDevice, h->stream);
  if (e == cudaSuccess && T) {
    ++h->launches;
    k_concat_rows<<<blocks_for(T * kTileRows, 256), 256, 0, h->stream>>>(
        a->tile_rows, a->num_tiles * kTileRows, b->tile_rows, b->num_tiles * kTileRows, static_cast<int32_t>(a->n_out),
        km->tile_rows);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    ++h->launches;
    k_concat_counters<<<1, 32, 0, h->stream>>>(a->counters, a->err, b->counters, b->err, km->counters, km->err);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    free_kmap(h, km);
    return cuda_error(h, e, "concat maps");
  }
  const sc_status st2 = build_group_orders(h, km);
  if (st2 != SC_OK) {
    free_kmap(h, km);
    return st2;
  }
  *out = km;
  return SC_OK;
}

}  // namespace sc
