// Neighbour-map build that allocates no device memory.
//
// Some callers cannot let a library allocate device memory: a host runtime
// that budgets every byte of device memory itself (an application embedding
// this library next to its own fixed-size pool, where an extra allocation could
// fail or push its data out), or a latency-sensitive path where growing an
// allocator pool would block on the driver.  For them this file provides one
// entry point whose only scratch is a file-scope __device__ array of fixed
// size; the caller passes the coordinates and the output map.
//
// Limits and behaviour:
//   * at most kNoAllocMaxVoxels (131072) voxels per call; larger inputs are
//     rejected with SC_EINVAL before any work is enqueued;
//   * the scratch (an 8 MiB hash table plus a status word) lives on every GPU
//     that loads the library, for the life of the process;
//   * every call shares that scratch and leaves the last call's contents in it;
//     each call clears the part it uses first, so calls that overlap on the GPU
//     (different streams or threads at the same time) race on it and must be
//     ordered by the caller;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it;
//   * every call waits for its own build (it reads the status word back), so
//     no call can be part of a CUDA graph: a call made while the handle's
//     stream is being captured is rejected with SC_EINVAL before it enqueues
//     anything.
#include "sc_common.cuh"
#include "sc_internal.h"

#include <mutex>

namespace sc {
namespace {

constexpr uint32_t kNoAllocSlots = 1u << 19;                  // 16-byte slots: 8 MiB
constexpr int64_t kNoAllocMaxVoxels = kNoAllocSlots / 4;     // load factor <= 1/4
constexpr int kNoAllocMaxDevices = 64;
constexpr unsigned long long kNaEmpty = ~0ull;

struct __align__(16) NaSlot {
  unsigned long long key;
  int val;
  int pad;
};

// The scratch.  In host code these names are host-side stand-ins, not device
// addresses; only the addresses returned by cudaGetSymbolAddress are passed to
// kernels.
static __device__ __align__(256) NaSlot g_na_slots[kNoAllocSlots];
static __device__ __align__(256) int g_na_status[64];

struct NaDevice {
  std::once_flag once;
  cudaError_t setup = cudaSuccess;
  NaSlot* slots = nullptr;
  int* status = nullptr;
};
NaDevice g_na_dev[kNoAllocMaxDevices];

// Looks up the scratch addresses on `device` (which must be current).
cudaError_t na_setup(int device, NaSlot** slots, int** status) {
  if (device < 0 || device >= kNoAllocMaxDevices) return cudaErrorInvalidDevice;
  NaDevice& d = g_na_dev[device];
  std::call_once(d.once, [&d]() {
    void* p = nullptr;
    d.setup = cudaGetSymbolAddress(&p, g_na_slots);
    if (d.setup != cudaSuccess) return;
    d.slots = static_cast<NaSlot*>(p);
    d.setup = cudaGetSymbolAddress(&p, g_na_status);
    if (d.setup != cudaSuccess) return;
    d.status = static_cast<int*>(p);
  });
  *slots = d.slots;
  *status = d.status;
  return d.setup;
}

__device__ __forceinline__ unsigned long long na_key(int b, int x, int y, int z) {
  return (static_cast<unsigned long long>(b) << 48) | (static_cast<unsigned long long>(x) << 32) |
         (static_cast<unsigned long long>(y) << 16) | static_cast<unsigned long long>(z);
}

// 64-bit finaliser fmix64 of MurmurHash3 (A. Appleby, public domain),
// folded to 32 bits.
__device__ __forceinline__ uint32_t na_hash(unsigned long long k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return static_cast<uint32_t>(k);
}

__device__ __forceinline__ bool na_coord_ok(int4 c) {
  return static_cast<unsigned>(c.x) <= 32767u && static_cast<unsigned>(c.y) <= 65535u &&
         static_cast<unsigned>(c.z) <= 65535u && static_cast<unsigned>(c.w) <= 65535u;
}

__global__ void k_na_insert(const int4* __restrict__ coords, int64_t n, NaSlot* slots, uint32_t mask, int* status) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  const int4 c = coords[i];
  if (!na_coord_ok(c)) {
    record_error(status, SC_ERANGE);
    return;
  }
  const unsigned long long key = na_key(c.x, c.y, c.z, c.w);
  uint32_t pos = na_hash(key) & mask;
  for (uint32_t it = 0; it <= mask; ++it) {
    const unsigned long long prev = atomicCAS(&slots[pos].key, kNaEmpty, key);
    if (prev == kNaEmpty) {
      slots[pos].val = static_cast<int>(i);
      return;
    }
    if (prev == key) {
      record_error(status, SC_EDUP_COORD);
      return;
    }
    pos = (pos + 1) & mask;
  }
  record_error(status, SC_ENOMEM);
}

// One thread per (voxel, offset): map_out[i*27 + v].
__global__ void k_na_probe(const int4* __restrict__ coords, int64_t n, const NaSlot* __restrict__ slots,
                           uint32_t mask, int dil, int32_t* __restrict__ map_out) {
  const int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (e >= n * 27) return;
  const int64_t i = e / 27;
  const int v = static_cast<int>(e - i * 27);
  const int4 c = coords[i];
  int r = -1;
  if (v == 13) {
    r = static_cast<int>(i);
  } else if (na_coord_ok(c)) {
    const int x = c.y + (v / 9 - 1) * dil, y = c.z + ((v / 3) % 3 - 1) * dil, z = c.w + (v % 3 - 1) * dil;
    if (static_cast<unsigned>(x) <= 65535u && static_cast<unsigned>(y) <= 65535u &&
        static_cast<unsigned>(z) <= 65535u) {
      const unsigned long long q = na_key(c.x, x, y, z);
      uint32_t pos = na_hash(q) & mask;
      for (uint32_t it = 0; it <= mask; ++it) {
        const ulonglong2 s = __ldg(reinterpret_cast<const ulonglong2*>(slots) + pos);
        if (s.x == q) {
          r = static_cast<int>(static_cast<uint32_t>(s.y));
          break;
        }
        if (s.x == kNaEmpty) break;
        pos = (pos + 1) & mask;
      }
    }
  }
  map_out[e] = r;
}

}  // namespace

sc_status build_subm_noalloc(Handle* h, const int32_t* coords, int64_t n, int dilation, int32_t* map_out) {
  if (n > kNoAllocMaxVoxels)
    return set_error(h, SC_EINVAL,
                     "sc_kmap_build_noalloc: n exceeds the fixed scratch limit of 131072 voxels; "
                     "use sc_kmap_build for larger inputs");
  cudaStreamCaptureStatus cap_st = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(h->stream, &cap_st);
  if (e != cudaSuccess) return cuda_error(h, e, "sc_kmap_build_noalloc: capture query");
  if (cap_st != cudaStreamCaptureStatusNone)
    return set_error(h, SC_EINVAL,
                     "sc_kmap_build_noalloc waits for its build on the handle's stream and cannot be called "
                     "while that stream is being captured");
  NaSlot* slots = nullptr;
  int* status = nullptr;
  e = na_setup(h->device, &slots, &status);
  if (e != cudaSuccess) return cuda_error(h, e, "sc_kmap_build_noalloc: cudaGetSymbolAddress");
  if (n == 0) return SC_OK;
  uint32_t cap = 1024;
  while (cap < 4 * static_cast<uint64_t>(n)) cap <<= 1;
  e = cudaMemsetAsync(slots, 0xFF, sizeof(NaSlot) * cap, h->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(status, 0, sizeof(int), h->stream);
  if (e != cudaSuccess) return cuda_error(h, e, "sc_kmap_build_noalloc: clear scratch");
  const int4* c4 = reinterpret_cast<const int4*>(coords);
  ++h->launches;
  k_na_insert<<<static_cast<unsigned>((n + 255) / 256), 256, 0, h->stream>>>(c4, n, slots, cap - 1, status);
  ++h->launches;
  k_na_probe<<<static_cast<unsigned>((n * 27 + 255) / 256), 256, 0, h->stream>>>(c4, n, slots, cap - 1, dilation,
                                                                                  map_out);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(h, e, "sc_kmap_build_noalloc: launch");
  int err = 0;
  e = cudaMemcpyAsync(&err, status, sizeof(int), cudaMemcpyDeviceToHost, h->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) return cuda_error(h, e, "sc_kmap_build_noalloc: status");
  if (err == SC_EDUP_COORD) return set_error(h, SC_EDUP_COORD, "duplicate coordinate (b, x, y, z)");
  if (err == SC_ERANGE)
    return set_error(h, SC_ERANGE, "coordinate out of range (b in [0, 32767], x/y/z in [0, 65535])");
  if (err != 0) return set_error(h, static_cast<sc_status>(err), "sc_kmap_build_noalloc failed");
  return SC_OK;
}

}  // namespace sc
