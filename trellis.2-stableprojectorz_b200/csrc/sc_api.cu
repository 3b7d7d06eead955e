// C ABI of libsparseconv_b200.so (declared in include/sparse_conv_b200.h).
//
// Every entry point validates its arguments, binds the handle's device for
// the duration of the call, enqueues on the handle's stream and returns a
// status code; nothing throws across the boundary.
#include "sc_common.cuh"
#include "sc_internal.h"

#include <cstdio>
#include <cstring>
#include <new>

namespace sc {

struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

sc_status set_error(Handle* h, sc_status st, const std::string& msg) {
  if (h) h->last_error = msg;
  return st;
}

sc_status cuda_error(Handle* h, cudaError_t e, const char* what) {
  char buf[512];
  snprintf(buf, sizeof(buf), "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
  if (e == cudaErrorMemoryAllocation) return set_error(h, SC_ENOMEM, buf);
  return set_error(h, SC_ECUDA, buf);
}

cudaError_t dev_alloc(Handle* h, void** p, size_t bytes) {
  return cudaMallocAsync(p, bytes ? bytes : 16, h->stream);
}

void dev_free(Handle* h, void* p) {
  if (p) cudaFreeAsync(p, h->stream);
}

}  // namespace sc

using sc::Handle;
using sc::KMap;

struct sc_handle {
  Handle impl;
};
struct sc_kmap {
  KMap* impl;
};

namespace {
sc_status device_status(Handle* h, const KMap* km) {
  int err = 0;
  cudaError_t e = cudaMemcpyAsync(&err, km->err, sizeof(int), cudaMemcpyDeviceToHost, h->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) return sc::cuda_error(h, e, "kmap status");
  switch (err) {
    case 0: return SC_OK;
    case SC_EDUP_COORD: return sc::set_error(h, SC_EDUP_COORD, "duplicate coordinate (b, x, y, z)");
    case SC_ERANGE: return sc::set_error(h, SC_ERANGE, "coordinate out of range (b in [0, 32767], x/y/z in [0, 65535])");
    case SC_ETIMEOUT: return sc::set_error(h, SC_ETIMEOUT, "device wait limit expired during map build");
    case SC_ENOMEM: return sc::set_error(h, SC_ENOMEM, "hash table overflow");
    default: return sc::set_error(h, static_cast<sc_status>(err), "kmap build failed");
  }
}

sc_status wrap_kmap(Handle* h, KMap* km, uint32_t flags, sc_kmap** out) {
  sc_kmap* w = new (std::nothrow) sc_kmap{km};
  if (!w) {
    sc::free_kmap(h, km);
    return sc::set_error(h, SC_ENOMEM, "host allocation failed");
  }
  if (!(flags & SC_BUILD_DEFER_CHECK)) {
    const sc_status st = device_status(h, km);
    if (st != SC_OK) {
      sc::free_kmap(h, km);
      delete w;
      return st;
    }
  }
  *out = w;
  return SC_OK;
}
}  // namespace

extern "C" {

const char* sc_version(void) { return "sparseconv_b200 0.1.0 (sm_100a)"; }

void sc_config_default(sc_config* cfg) {
  if (!cfg) return;
  std::memset(cfg, 0, sizeof(*cfg));
  cfg->device = 0;
  cfg->map_mode = SC_MAP_HASH;
}

sc_status sc_create(sc_handle** out, const sc_config* cfg) {
  if (!out) return SC_EINVAL;
  *out = nullptr;
  sc_config c;
  sc_config_default(&c);
  if (cfg) c = *cfg;
  if (c.map_mode != SC_MAP_HASH && c.map_mode != SC_MAP_SORT) return SC_EINVAL;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || c.device < 0 || c.device >= ndev) return SC_ECUDA;
  sc_handle* h = new (std::nothrow) sc_handle();
  if (!h) return SC_ENOMEM;
  h->impl.device = c.device;
  h->impl.map_mode = c.map_mode;
  h->impl.debug_bounds = c.debug_bounds;
  sc::DeviceGuard g(c.device);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, c.device) != cudaSuccess || prop.major < 10) {
    delete h;
    return SC_EUNSUPPORTED;
  }
  h->impl.num_sms = prop.multiProcessorCount;
  // The zeroing runs on the legacy stream; wait for it so that kernels on a
  // non-blocking caller stream never see the error word before it is zero.
  if (cudaMalloc(reinterpret_cast<void**>(&h->impl.derr), 16) != cudaSuccess ||
      cudaMemset(h->impl.derr, 0, 16) != cudaSuccess || cudaStreamSynchronize(cudaStreamLegacy) != cudaSuccess) {
    if (h->impl.derr) cudaFree(h->impl.derr);
    delete h;
    return SC_ECUDA;
  }
  // Keep freed stream-ordered allocations cached in the pool (best effort:
  // without it the pool only releases memory sooner).
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, c.device) == cudaSuccess) {
    uint64_t thr = ~0ull;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
  }
  *out = h;
  return SC_OK;
}

sc_status sc_destroy(sc_handle* h) {
  if (!h) return SC_EINVAL;
  {
    sc::DeviceGuard g(h->impl.device);
    cudaStreamSynchronize(h->impl.stream);
    if (h->impl.derr) cudaFree(h->impl.derr);
    if (h->impl.push_ticket) cudaFree(h->impl.push_ticket);
  }
  delete h;
  return SC_OK;
}

sc_status sc_peer_alloc(sc_handle* h, size_t bytes, void** ptr, void* ipc_handle_out) {
  if (!h || !ptr || !ipc_handle_out) return SC_EINVAL;
  if (bytes == 0) return sc::set_error(&h->impl, SC_EINVAL, "peer buffer size must be positive");
  sc::DeviceGuard g(h->impl.device);
  return sc::peer_alloc(&h->impl, bytes, ptr, ipc_handle_out);
}

sc_status sc_peer_free(sc_handle* h, void* ptr) {
  if (!h) return SC_EINVAL;
  sc::DeviceGuard g(h->impl.device);
  if (ptr) {
    const cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) return sc::cuda_error(&h->impl, e, "free peer buffer");
  }
  return SC_OK;
}

sc_status sc_peer_open(sc_handle* h, const void* ipc_handle, void** peer_ptr) {
  if (!h || !ipc_handle || !peer_ptr) return SC_EINVAL;
  sc::DeviceGuard g(h->impl.device);
  return sc::peer_open(&h->impl, ipc_handle, peer_ptr);
}

sc_status sc_peer_close(sc_handle* h, void* peer_ptr) {
  if (!h) return SC_EINVAL;
  sc::DeviceGuard g(h->impl.device);
  if (peer_ptr) {
    const cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
    if (e != cudaSuccess) return sc::cuda_error(&h->impl, e, "close peer buffer");
  }
  return SC_OK;
}

sc_status sc_halo_push(sc_handle* h, const void* feats, int32_t row_bytes, const int32_t* src_row,
                       const int32_t* dst_peer, const int64_t* dst_off, int64_t n_send, void* const* peer_bufs,
                       uint32_t* const* peer_flags, int32_t world, int32_t rank, uint32_t epoch) {
  if (!h) return SC_EINVAL;
  Handle* H = &h->impl;
  if (world < 2 || world > 32 || rank < 0 || rank >= world)
    return sc::set_error(H, SC_EINVAL, "halo push: need 2 <= world <= 32 and 0 <= rank < world");
  if (row_bytes <= 0 || row_bytes % 16 != 0) return sc::set_error(H, SC_EINVAL, "row_bytes must be a multiple of 16");
  if (n_send < 0) return sc::set_error(H, SC_EINVAL, "n_send must be >= 0");
  if (!peer_bufs || !peer_flags || (n_send > 0 && (!feats || !src_row || !dst_peer || !dst_off)) ||
      !sc::aligned(feats, 16))
    return sc::set_error(H, SC_EINVAL, "halo push: missing or misaligned device arrays");
  sc::DeviceGuard g(H->device);
  return sc::halo_push(H, feats, row_bytes, src_row, dst_peer, dst_off, n_send, peer_bufs, peer_flags, world, rank,
                       epoch);
}

sc_status sc_halo_wait(sc_handle* h, const uint32_t* flags, int32_t world, int32_t rank, uint32_t epoch) {
  if (!h) return SC_EINVAL;
  Handle* H = &h->impl;
  if (world < 2 || world > 32 || rank < 0 || rank >= world || !flags || !sc::aligned(flags, 4))
    return sc::set_error(H, SC_EINVAL, "halo wait: need 2 <= world <= 32, 0 <= rank < world and 4-byte aligned flags");
  sc::DeviceGuard g(H->device);
  return sc::halo_wait(H, flags, world, rank, epoch);
}

sc_status sc_set_conv_ctas(sc_handle* h, int32_t max_ctas) {
  if (!h) return SC_EINVAL;
  if (max_ctas < 0) return sc::set_error(&h->impl, SC_EINVAL, "max_ctas must be >= 0");
  h->impl.conv_ctas = max_ctas;
  return SC_OK;
}

sc_status sc_set_stream(sc_handle* h, void* stream) {
  if (!h) return SC_EINVAL;
  h->impl.stream = static_cast<cudaStream_t>(stream);
  return SC_OK;
}

sc_status sc_synchronize(sc_handle* h) {
  if (!h) return SC_EINVAL;
  sc::DeviceGuard g(h->impl.device);
  Handle* H = &h->impl;
  int err = 0;
  cudaError_t e = cudaMemcpyAsync(&err, H->derr, sizeof(int), cudaMemcpyDeviceToHost, H->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(H->stream);
  if (e != cudaSuccess) return sc::cuda_error(H, e, "synchronize");
  if (err != 0) {
    cudaMemsetAsync(H->derr, 0, sizeof(int), H->stream);
    cudaStreamSynchronize(H->stream);
    return sc::set_error(H, static_cast<sc_status>(err),
                         err == SC_ETIMEOUT ? "device wait limit expired in a conv kernel"
                         : err == SC_EINVAL ? "a kernel rejected an argument (halo push destination out of range or "
                                              "not 16-byte aligned)"
                                            : "conv kernel error");
  }
  return SC_OK;
}

const char* sc_last_error(const sc_handle* h) {
  if (!h) return "null handle";
  return h->impl.last_error.c_str();
}

uint64_t sc_launch_count(const sc_handle* h) { return h ? h->impl.launches : 0; }

sc_status sc_kmap_build(sc_handle* h, const int32_t* coords, int64_t n, int32_t kernel_size, int32_t dilation,
                        uint32_t flags, sc_kmap** out) {
  if (!h || !out) return SC_EINVAL;
  *out = nullptr;
  Handle* H = &h->impl;
  if (n < 0 || n >= (1ll << 29)) return sc::set_error(H, SC_EINVAL, "n must be in [0, 2^29)");
  if (n > 0 && (!coords || !sc::aligned(coords, 16)))
    return sc::set_error(H, SC_EINVAL, "coords must be a 16-byte aligned device pointer");
  if (kernel_size != 3) return sc::set_error(H, SC_EUNSUPPORTED, "only 3x3x3 submanifold kernels");
  if (dilation < 1 || dilation > 1024) return sc::set_error(H, SC_EINVAL, "dilation must be in [1, 1024]");
  sc::DeviceGuard g(H->device);
  KMap* km = nullptr;
  const sc_status st = sc::build_subm(H, coords, n, 0, n, sc::Dil{dilation, dilation, dilation}, flags, &km);
  if (st != SC_OK) return st;
  return wrap_kmap(H, km, flags, out);
}

sc_status sc_kmap_build_dilated(sc_handle* h, const int32_t* coords, int64_t n_in, int64_t out_begin,
                                int64_t out_end, int32_t dil_x, int32_t dil_y, int32_t dil_z, uint32_t flags,
                                sc_kmap** out) {
  if (!h || !out) return SC_EINVAL;
  *out = nullptr;
  Handle* H = &h->impl;
  if (n_in < 0 || n_in >= (1ll << 29)) return sc::set_error(H, SC_EINVAL, "n_in must be in [0, 2^29)");
  if (out_begin < 0 || out_end < out_begin || out_end > n_in)
    return sc::set_error(H, SC_EINVAL, "need 0 <= out_begin <= out_end <= n_in");
  if (n_in > 0 && (!coords || !sc::aligned(coords, 16)))
    return sc::set_error(H, SC_EINVAL, "coords must be a 16-byte aligned device pointer");
  for (const int32_t d : {dil_x, dil_y, dil_z})
    if (d < 1 || d > 1024) return sc::set_error(H, SC_EINVAL, "every dilation must be in [1, 1024]");
  sc::DeviceGuard g(H->device);
  KMap* km = nullptr;
  const sc_status st =
      sc::build_subm(H, coords, n_in, out_begin, out_end - out_begin, sc::Dil{dil_x, dil_y, dil_z}, flags, &km);
  if (st != SC_OK) return st;
  return wrap_kmap(H, km, flags, out);
}

sc_status sc_kmap_build_range(sc_handle* h, const int32_t* coords, int64_t n_in, int64_t out_begin, int64_t out_end,
                              int32_t kernel_size, int32_t dilation, uint32_t flags, sc_kmap** out) {
  if (!h || !out) return SC_EINVAL;
  *out = nullptr;
  if (kernel_size != 3) return sc::set_error(&h->impl, SC_EUNSUPPORTED, "only 3x3x3 submanifold kernels");
  return sc_kmap_build_dilated(h, coords, n_in, out_begin, out_end, dilation, dilation, dilation, flags, out);
}

sc_status sc_kmap_build_ex(sc_handle* h, const int32_t* coords, int64_t n_in, int64_t n_out, int32_t kernel_size,
                           int32_t dilation, uint32_t flags, sc_kmap** out) {
  if (h && (n_out < 0 || n_out > n_in)) return sc::set_error(&h->impl, SC_EINVAL, "n_out must be in [0, n_in]");
  return sc_kmap_build_range(h, coords, n_in, 0, n_out, kernel_size, dilation, flags, out);
}

sc_status sc_kmap_concat(sc_handle* h, const sc_kmap* first, const sc_kmap* second, uint32_t flags, sc_kmap** out) {
  if (!h || !out || !first || !second) return SC_EINVAL;
  *out = nullptr;
  Handle* H = &h->impl;
  sc::DeviceGuard g(H->device);
  KMap* km = nullptr;
  const sc_status st = sc::concat_maps(H, first->impl, second->impl, &km);
  if (st != SC_OK) return st;
  return wrap_kmap(H, km, flags, out);
}

sc_status sc_kmap_build_down2(sc_handle* h, const int32_t* coords, int64_t n, uint32_t flags, sc_kmap** out) {
  if (!h || !out) return SC_EINVAL;
  *out = nullptr;
  Handle* H = &h->impl;
  if (n < 0 || n >= (1ll << 28)) return sc::set_error(H, SC_EINVAL, "n must be in [0, 2^28)");
  if (n > 0 && (!coords || !sc::aligned(coords, 16)))
    return sc::set_error(H, SC_EINVAL, "coords must be a 16-byte aligned device pointer");
  sc::DeviceGuard g(H->device);
  KMap* km = nullptr;
  const sc_status st = sc::build_down2(H, coords, n, flags, &km);
  if (st != SC_OK) return st;
  return wrap_kmap(H, km, flags, out);
}

sc_status sc_kmap_build_up2(sc_handle* h, const sc_kmap* down, uint32_t flags, sc_kmap** out) {
  if (!h || !out || !down) return SC_EINVAL;
  *out = nullptr;
  Handle* H = &h->impl;
  sc::DeviceGuard g(H->device);
  KMap* km = nullptr;
  const sc_status st = sc::build_up2(H, down->impl, flags, &km);
  if (st != SC_OK) return st;
  return wrap_kmap(H, km, flags, out);
}

sc_status sc_kmap_build_noalloc(sc_handle* h, const int32_t* coords, int64_t n, int32_t dilation,
                                int32_t* map_out) {
  if (!h) return SC_EINVAL;
  Handle* H = &h->impl;
  if (n < 0) return sc::set_error(H, SC_EINVAL, "n must be >= 0");
  if (n > 0 && (!coords || !sc::aligned(coords, 16) || !map_out || !sc::aligned(map_out, 4)))
    return sc::set_error(H, SC_EINVAL, "coords (16-byte aligned) and map_out must be device pointers");
  if (dilation < 1 || dilation > 1024) return sc::set_error(H, SC_EINVAL, "dilation must be in [1, 1024]");
  sc::DeviceGuard g(H->device);
  return sc::build_subm_noalloc(H, coords, n, dilation, map_out);
}

sc_status sc_kmap_out_coords(sc_handle* h, const sc_kmap* km, int32_t* coords_out) {
  if (!h || !km) return SC_EINVAL;
  Handle* H = &h->impl;
  if (km->impl->kind != SC_KMAP_DOWN2 || !km->impl->out_coords)
    return sc::set_error(H, SC_EINVAL, "only down2 maps have new coords");
  if (km->impl->n_out == 0) return SC_OK;
  if (!coords_out) return sc::set_error(H, SC_EINVAL, "null output");
  sc::DeviceGuard g(H->device);
  cudaError_t e = cudaMemcpyAsync(coords_out, km->impl->out_coords, sizeof(int32_t) * 4 * km->impl->n_out,
                                  cudaMemcpyDeviceToDevice, H->stream);
  return e == cudaSuccess ? SC_OK : sc::cuda_error(H, e, "copy out coords");
}

sc_status sc_kmap_export(sc_handle* h, const sc_kmap* km, int32_t* map_out) {
  if (!h || !km) return SC_EINVAL;
  Handle* H = &h->impl;
  if (km->impl->n_out > 0 && !map_out) return sc::set_error(H, SC_EINVAL, "null output");
  sc::DeviceGuard g(H->device);
  return sc::export_map(H, km->impl, map_out);
}

sc_status sc_kmap_get_info(sc_handle* h, const sc_kmap* km, sc_kmap_info* info) {
  if (!h || !km || !info) return SC_EINVAL;
  Handle* H = &h->impl;
  sc::DeviceGuard g(H->device);
  unsigned long long c[3] = {0, 0, 0};
  cudaError_t e = cudaMemcpyAsync(c, km->impl->counters, sizeof(c), cudaMemcpyDeviceToHost, H->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(H->stream);
  if (e != cudaSuccess) return sc::cuda_error(H, e, "kmap info");
  info->kind = km->impl->kind;
  info->kernel_volume = km->impl->K;
  info->n_in = km->impl->n_in;
  info->n_out = km->impl->n_out;
  info->num_pairs = static_cast<int64_t>(c[0]);
  info->num_tiles = km->impl->num_tiles;
  info->tile_pairs = static_cast<int64_t>(c[1]);
  info->halo_max = km->impl->lidx ? static_cast<int64_t>(c[2]) : -1;
  return SC_OK;
}

sc_status sc_kmap_check(sc_handle* h, const sc_kmap* km) {
  if (!h || !km) return SC_EINVAL;
  sc::DeviceGuard g(h->impl.device);
  return device_status(&h->impl, km->impl);
}

sc_status sc_kmap_free(sc_handle* h, sc_kmap* km) {
  if (!h || !km) return SC_EINVAL;
  sc::DeviceGuard g(h->impl.device);
  sc::free_kmap(&h->impl, km->impl);
  delete km;
  return SC_OK;
}

namespace {

sc_status conv3d_impl(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight, const void* bias,
                      const void* residual, void* out, int32_t ci, int32_t co, sc_dtype dtype, uint32_t epilogue,
                      float ln_eps, const sc::ConvWait& wait) {
  if (!h || !km) return SC_EINVAL;
  Handle* H = &h->impl;
  const KMap* K = km->impl;
  if (ci <= 0 || co <= 0) return sc::set_error(H, SC_EINVAL, "channel counts must be positive");
  if (epilogue & ~(SC_EPI_SILU | SC_EPI_RESIDUAL | SC_EPI_LAYERNORM))
    return sc::set_error(H, SC_EINVAL, "unknown epilogue flag");
  if (dtype != SC_F32 && dtype != SC_BF16 && dtype != SC_F16) return sc::set_error(H, SC_EINVAL, "unknown dtype");
  sc::DeviceGuard g(H->device);
  if (K->n_out == 0) return wait.flags ? sc::halo_wait(H, wait.flags, wait.world, wait.rank, wait.epoch) : SC_OK;
  if (!weight || !out || (K->n_in > 0 && !feats)) return sc::set_error(H, SC_EINVAL, "null operand");
  if ((epilogue & SC_EPI_RESIDUAL) && !residual) return sc::set_error(H, SC_EINVAL, "residual missing");
  if (!(ln_eps >= 0.f)) return sc::set_error(H, SC_EINVAL, "ln_eps must be >= 0");
  if (dtype == SC_F32) {
    if (wait.flags) {
      const sc_status st = sc::halo_wait(H, wait.flags, wait.world, wait.rank, wait.epoch);
      if (st != SC_OK) return st;
    }
    return sc::conv_simt_f32(H, K, static_cast<const float*>(feats), static_cast<const float*>(weight),
                             static_cast<const float*>(bias), static_cast<const float*>(residual),
                             static_cast<float*>(out), ci, co, epilogue, ln_eps);
  }
  return sc::conv_tc(H, K, feats, weight, bias, residual, out, ci, co, dtype, epilogue, ln_eps, wait);
}

}  // namespace

sc_status sc_conv3d(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight, const void* bias,
                    const void* residual, void* out, int32_t ci, int32_t co, sc_dtype dtype, uint32_t epilogue,
                    float ln_eps) {
  return conv3d_impl(h, km, feats, weight, bias, residual, out, ci, co, dtype, epilogue, ln_eps, sc::ConvWait());
}

sc_status sc_conv3d_halo(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight, const void* bias,
                         const void* residual, void* out, int32_t ci, int32_t co, sc_dtype dtype, uint32_t epilogue,
                         float ln_eps, const uint32_t* flags, int32_t world, int32_t rank, uint32_t epoch) {
  if (!h || !km) return SC_EINVAL;
  if (world < 2 || world > 32 || rank < 0 || rank >= world || !flags || !sc::aligned(flags, 4))
    return sc::set_error(&h->impl, SC_EINVAL,
                         "conv halo wait: need 2 <= world <= 32, 0 <= rank < world and 4-byte aligned flags");
  if (km->impl->kind != SC_KMAP_SUBM) return sc::set_error(&h->impl, SC_EINVAL, "map is not a submanifold map");
  sc::ConvWait w;
  w.flags = flags;
  w.world = world;
  w.rank = rank;
  w.epoch = epoch;
  return conv3d_impl(h, km, feats, weight, bias, residual, out, ci, co, dtype, epilogue, ln_eps, w);
}

sc_status sc_conv3d_subm(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight, const void* bias,
                         const void* residual, void* out, int32_t ci, int32_t co, sc_dtype dtype, uint32_t epilogue,
                         float ln_eps) {
  if (!h || !km) return SC_EINVAL;
  if (km->impl->kind != SC_KMAP_SUBM) return sc::set_error(&h->impl, SC_EINVAL, "map is not a submanifold map");
  return sc_conv3d(h, km, feats, weight, bias, residual, out, ci, co, dtype, epilogue, ln_eps);
}

sc_status sc_conv3d_down2(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight, const void* bias,
                          void* out, int32_t ci, int32_t co, sc_dtype dtype, uint32_t epilogue) {
  if (!h || !km) return SC_EINVAL;
  if (km->impl->kind != SC_KMAP_DOWN2) return sc::set_error(&h->impl, SC_EINVAL, "map is not a down2 map");
  if (epilogue & (SC_EPI_RESIDUAL | SC_EPI_LAYERNORM)) return sc::set_error(&h->impl, SC_EINVAL, "SiLU only");
  return sc_conv3d(h, km, feats, weight, bias, nullptr, out, ci, co, dtype, epilogue, 0.f);
}

sc_status sc_conv3d_up2(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight, const void* bias,
                        void* out, int32_t ci, int32_t co, sc_dtype dtype, uint32_t epilogue) {
  if (!h || !km) return SC_EINVAL;
  if (km->impl->kind != SC_KMAP_UP2) return sc::set_error(&h->impl, SC_EINVAL, "map is not an up2 map");
  if (epilogue & (SC_EPI_RESIDUAL | SC_EPI_LAYERNORM)) return sc::set_error(&h->impl, SC_EINVAL, "SiLU only");
  return sc_conv3d(h, km, feats, weight, bias, nullptr, out, ci, co, dtype, epilogue, 0.f);
}

sc_status sc_conv3d_depthwise(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight,
                              const void* bias, void* out, int32_t channels, sc_dtype dtype) {
  if (!h || !km) return SC_EINVAL;
  Handle* H = &h->impl;
  const KMap* K = km->impl;
  if (K->kind != SC_KMAP_SUBM || K->K != 27) return sc::set_error(H, SC_EINVAL, "map is not a 3x3x3 submanifold map");
  if (dtype != SC_F32 && dtype != SC_BF16 && dtype != SC_F16) return sc::set_error(H, SC_EINVAL, "unknown dtype");
  if (channels <= 0 || channels % 8 != 0)
    return sc::set_error(H, SC_EINVAL, "depthwise conv needs a positive channel count that is a multiple of 8");
  if (K->n_out == 0) return SC_OK;
  if (!weight || !out || (K->n_in > 0 && !feats)) return sc::set_error(H, SC_EINVAL, "null operand");
  if (!sc::aligned(feats, 16) || !sc::aligned(out, 16))
    return sc::set_error(H, SC_EINVAL, "feats and out must be 16-byte aligned");
  sc::DeviceGuard g(H->device);
  return sc::conv_depthwise(H, K, feats, weight, bias, out, channels, dtype);
}

sc_status sc_subdivide2(sc_handle* h, const int32_t* coords, int64_t n, const uint8_t* child_mask,
                        const void* feats, int32_t row_bytes, int32_t* out_coords, int32_t* out_parent,
                        void* out_feats, int64_t capacity, int64_t* n_out) {
  if (!h) return SC_EINVAL;
  Handle* H = &h->impl;
  if (!n_out) return sc::set_error(H, SC_EINVAL, "null n_out");
  *n_out = 0;
  if (n < 0 || n >= (1ll << 28)) return sc::set_error(H, SC_EINVAL, "n must be in [0, 2^28)");
  if (n > 0 && (!coords || !sc::aligned(coords, 16)))
    return sc::set_error(H, SC_EINVAL, "coords must be a 16-byte aligned device pointer");
  if (out_coords && !sc::aligned(out_coords, 16))
    return sc::set_error(H, SC_EINVAL, "out_coords must be 16-byte aligned");
  if (out_feats) {
    if (!out_coords || !out_parent || (n > 0 && !feats))
      return sc::set_error(H, SC_EINVAL, "copying features needs feats, out_coords and out_parent");
    if (row_bytes <= 0 || row_bytes % 16 != 0) return sc::set_error(H, SC_EINVAL, "row_bytes must be a multiple of 16");
    if (!sc::aligned(out_feats, 16) || (feats && !sc::aligned(feats, 16)))
      return sc::set_error(H, SC_EINVAL, "feats and out_feats must be 16-byte aligned");
  }
  if (capacity < 0) return sc::set_error(H, SC_EINVAL, "capacity must be >= 0");
  if (n == 0) return SC_OK;
  sc::DeviceGuard g(H->device);
  return sc::subdivide2(H, coords, n, child_mask, feats, row_bytes, out_coords, out_parent, out_feats, capacity,
                        n_out);
}

sc_status sc_attention_varlen(sc_handle* h, const void* q, const void* k, const void* v, void* out,
                              const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_kv, int32_t batch,
                              int32_t num_heads, int32_t head_dim, float scale, sc_dtype dtype) {
  if (!h) return SC_EINVAL;
  Handle* H = &h->impl;
  if (head_dim != 64) return sc::set_error(H, SC_EUNSUPPORTED, "attention: head_dim must be 64");
  if (dtype != SC_BF16 && dtype != SC_F16) return sc::set_error(H, SC_EUNSUPPORTED, "attention: bf16 or f16 only");
  if (batch < 1 || num_heads < 1 || num_heads > 65535 || !cu_seqlens_q || !cu_seqlens_kv)
    return sc::set_error(H, SC_EINVAL, "attention: need batch >= 1, 1 <= num_heads <= 65535 and both cu_seqlens");
  if (cu_seqlens_q[0] != 0 || cu_seqlens_kv[0] != 0)
    return sc::set_error(H, SC_EINVAL, "attention: cu_seqlens must start at 0");
  for (int32_t b = 0; b < batch; ++b)
    if (cu_seqlens_q[b + 1] < cu_seqlens_q[b] || cu_seqlens_kv[b + 1] < cu_seqlens_kv[b])
      return sc::set_error(H, SC_EINVAL, "attention: cu_seqlens must be non-decreasing");
  if (!(scale > 0.f)) return sc::set_error(H, SC_EINVAL, "attention: scale must be positive");
  if (cu_seqlens_q[batch] == 0) return SC_OK;
  if (!q || !out || (cu_seqlens_kv[batch] > 0 && (!k || !v)))
    return sc::set_error(H, SC_EINVAL, "attention: null operand");
  if (!sc::aligned(q, 16) || !sc::aligned(out, 16) || (k && !sc::aligned(k, 16)) || (v && !sc::aligned(v, 16)))
    return sc::set_error(H, SC_EINVAL, "attention: q, k, v and out must be 16-byte aligned device arrays");
  sc::DeviceGuard g(H->device);
  return sc::attention_varlen(H, q, k, v, out, cu_seqlens_q, cu_seqlens_kv, batch, num_heads, scale, dtype);
}

sc_status sc_layernorm_silu(sc_handle* h, void* x, int64_t n, int32_t c, sc_dtype dtype, int32_t apply_silu,
                            float eps) {
  if (!h) return SC_EINVAL;
  Handle* H = &h->impl;
  if (n < 0 || c <= 0 || c > 4096 || (n > 0 && !x)) return sc::set_error(H, SC_EINVAL, "bad layernorm shape");
  if (n == 0) return SC_OK;
  sc::DeviceGuard g(H->device);
  return sc::layernorm_silu(H, x, n, c, dtype, apply_silu, eps);
}

}  // extern "C"
