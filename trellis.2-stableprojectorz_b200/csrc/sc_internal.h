// Internal structures shared by the engine's translation units.
#pragma once
#include <cstdint>
#include <string>
#include <cuda_runtime.h>
#include "../../include/sparse_conv_b200.h"

namespace sc {

// Output rows are processed in tiles of this many rows (one TMEM lane each).
constexpr int kTileRows = 128;
// Convs with fewer items (tile groups x output-channel blocks) per CTA than
// this take them in the map's work order; more items per CTA keep the
// natural tile order (already balanced, better L2 locality).
constexpr int64_t kWorkOrderMaxItemsPerCta = 64;

struct Handle {
  int device = 0;
  int map_mode = SC_MAP_HASH;
  int debug_bounds = 0;
  cudaStream_t stream = nullptr;
  int num_sms = 148;
  int conv_ctas = 0;  // CTAs of the tensor-core conv; 0 = one per SM
  void* push_ticket = nullptr;  // block ticket of the halo push kernel
  int* derr = nullptr;  // device error word written by conv kernels
  unsigned long long launches = 0;  // kernels this handle has launched
  std::string last_error;
};

// Neighbour / gather map in the layout the conv kernels consume.
//
//   tile_rows[t*128 + i]      output row handled by slot i of tile t (-1 = pad)
//   tile_mask[t]              bit v set when some row of tile t has offset v
//   gidx[(t*K + v)*128 + i]   input row gathered for slot i, offset v (-1 = none)
//
// Tiles are formed after sorting output rows by their K-bit neighbour mask
// (stable), so rows of one tile share most of their offsets.
constexpr int kHaloCap = 416;  // halo rows a tile may stage for the halo-staged conv

struct KMap {
  int kind = SC_KMAP_SUBM;
  int K = 27;
  int64_t n_in = 0;
  int64_t n_out = 0;
  int64_t num_tiles = 0;
  int32_t* gidx = nullptr;
  int32_t* tile_rows = nullptr;
  uint32_t* tile_mask = nullptr;
  // Groups of TPI = 1, 2, 4 consecutive tiles (index 0, 1, 2) ordered by
  // descending work (number of offsets the group runs); the conv schedules
  // its items in this order.  Built with the map, on its stream, when a conv
  // could use it (fewer than kWorkOrderMaxItemsPerCta * num_sms groups); null
  // otherwise.
  int32_t* group_order[3] = {nullptr, nullptr, nullptr};
  // Halo tiles (SC_BUILD_HALO): tiles are output rows in order; per tile the
  // distinct input rows its gathers read (kHaloCap slots, padded with -1 to a
  // multiple of 4) and per (tile, offset, slot) the position of the gathered
  // row in that list (0xFFFF = no neighbour).  A tile with more than
  // kHaloCap distinct rows is gathered straight from global memory by the
  // halo conv.  The largest halo is kept in counters[2].
  int32_t* halo_rows = nullptr;   // [num_tiles][kHaloCap]
  int32_t* halo_n = nullptr;      // [num_tiles]
  uint16_t* lidx = nullptr;       // [num_tiles][27][128]
  // Concatenated maps (concat_maps): tiles [split_tile, num_tiles) came from
  // the second map and are scheduled after every earlier tile; -1 = no split.
  int64_t split_tile = -1;
  int32_t* out_coords = nullptr;   // down-sample: parent coords [n_out, 4]
  int32_t* parent_of = nullptr;    // down-sample: parent of every fine row [n_in]
  unsigned long long* counters = nullptr;  // [0] valid pairs, [1] tile pairs
  int* err = nullptr;              // device error word of the build
};

// Helpers implemented in sc_api.cu
cudaError_t dev_alloc(Handle* h, void** p, size_t bytes);
void dev_free(Handle* h, void* p);

// Per-axis dilation of a 3x3x3 kernel (dilD on x, dilH on y, dilW on z).
struct Dil {
  int x, y, z;
};

// kmap construction (sc_kmap.cu)
sc_status build_subm(Handle* h, const int32_t* coords, int64_t n, int64_t out_begin, int64_t n_out, Dil dilation,
                     uint32_t flags, KMap** out);
sc_status build_down2(Handle* h, const int32_t* coords, int64_t n, uint32_t flags, KMap** out);
sc_status build_up2(Handle* h, const KMap* down, uint32_t flags, KMap** out);
sc_status export_map(Handle* h, const KMap* km, int32_t* map_out);
// allocation-free map build into caller memory (sc_noalloc.cu)
// peer-memory halo exchange
sc_status peer_alloc(Handle* h, size_t bytes, void** ptr, void* ipc_handle_out);
sc_status peer_open(Handle* h, const void* ipc_handle, void** peer_ptr);
sc_status halo_push(Handle* h, const void* feats, int row_bytes, const int32_t* src_row, const int32_t* dst_peer,
                    const int64_t* dst_off, int64_t n_send, void* const* peer_bufs, uint32_t* const* peer_flags,
                    int world, int rank, uint32_t epoch);
sc_status halo_wait(Handle* h, const uint32_t* flags, int world, int rank, uint32_t epoch);
sc_status concat_maps(Handle* h, const KMap* a, const KMap* b, KMap** out);
sc_status build_subm_noalloc(Handle* h, const int32_t* coords, int64_t n, int dilation, int32_t* map_out);
void free_kmap(Handle* h, KMap* km);

// A halo exchange the conv waits for on the device before it gathers halo
// rows: word r of `flags` must reach `epoch` for every r != rank.
struct ConvWait {
  const uint32_t* flags = nullptr;
  int world = 0;
  int rank = 0;
  uint32_t epoch = 0;
};

// conv launchers
sc_status conv_tc(Handle* h, const KMap* km, const void* feats, const void* weight, const void* bias,
                  const void* residual, void* out, int ci, int co, sc_dtype dtype, uint32_t epi, float eps,
                  const ConvWait& wait = ConvWait());
sc_status conv_simt_f32(Handle* h, const KMap* km, const float* feats, const float* weight, const float* bias,
                        const float* residual, float* out, int ci, int co, uint32_t epi, float eps);
sc_status check_gather_bounds(Handle* h, const KMap* km);
sc_status layernorm_silu(Handle* h, void* x, int64_t n, int c, sc_dtype dtype, int silu, float eps);
// variable-length attention, head dim 64 (sc_attn.cu); cu_q / cu_kv are host arrays
sc_status attention_varlen(Handle* h, const void* q, const void* k, const void* v, void* out, const int32_t* cu_q,
                           const int32_t* cu_kv, int batch, int heads, float scale, sc_dtype dtype);
// 2x2x2 subdivision with an optional child mask (sc_subdiv.cu)
sc_status subdivide2(Handle* h, const int32_t* coords, int64_t n, const uint8_t* child_mask, const void* feats,
                     int row_bytes, int32_t* out_coords, int32_t* out_parent, void* out_feats, int64_t capacity,
                     int64_t* n_out);
// depthwise 3x3x3 submanifold conv over a subm map (sc_conv_dw.cu)
sc_status conv_depthwise(Handle* h, const KMap* km, const void* feats, const void* weight, const void* bias,
                         void* out, int c, sc_dtype dtype);

// radix sort (sc_sort.cu): sorts (key, value) pairs on bits [begin_bit, end_bit)
size_t radix_sort_temp_bytes(int64_t n, int key_bytes, int passes);
sc_status radix_sort_pairs_u64(Handle* h, uint64_t* keys, uint32_t* vals, uint64_t* keys_alt, uint32_t* vals_alt,
                               int64_t n, int begin_bit, int end_bit, void* temp, size_t temp_bytes, int* err,
                               bool* result_in_alt);
// With hist_ready the caller has zeroed `temp` (radix_sort_temp_bytes) and
// added every key's digit counts into its first passes x kRadixBins words
// (pass p counts bits [begin_bit + 8p, begin_bit + 8p + 8)).
constexpr int kRadixBins = 256;
sc_status radix_sort_pairs_u32(Handle* h, uint32_t* keys, uint32_t* vals, uint32_t* keys_alt, uint32_t* vals_alt,
                               int64_t n, int begin_bit, int end_bit, void* temp, size_t temp_bytes, int* err,
                               bool* result_in_alt, bool hist_ready = false);

sc_status set_error(Handle* h, sc_status st, const std::string& msg);
sc_status cuda_error(Handle* h, cudaError_t e, const char* what);

}  // namespace sc
