/*
 * sparse_conv_b200.h -- C ABI of the B200 (sm_100a) submanifold sparse conv3d
 * engine (libsparseconv_b200.so).
 *
 * The library replaces the sparse-conv operator of TRELLIS.2:
 *   - TS/WebGPU port: SparseConv3d.forward(x: SparseTensor, ctx)
 *     (src/sparse/ops/conv3d.ts:41-222) with its three WGSL passes
 *     (src/sparse/ops/conv3d_wgsl.ts:44-231);
 *   - Python: the module selected by SPARSE_CONV_BACKEND under
 *     trellis2/modules/sparse/conv (conv_none.py + hashmap_fallback.py,
 *     README.md:27,109,111).
 *
 * Conventions (same operands as the reference):
 *   coords   int32 [N,4] rows (b, x, y, z), device memory, 16-byte aligned,
 *            0 <= b <= 32767, 0 <= x, y, z <= 65535
 *            (src/sparse/sparse_tensor.ts:19)
 *   feats    [N, Ci] row-major, dtype given per call
 *   weight   [Co, Kd, Kh, Kw, Ci] row-major (checkpoint layout,
 *            src/sparse/ops/conv3d.ts:5,19,48-49); 3x3x3 for submanifold,
 *            2x2x2 for the stride-2 down/up convolutions
 *   bias     [Co] in the feature dtype, or NULL (conv3d.ts:176-184)
 *   out      [N_out, Co] in the feature dtype
 * Kernel map: int32 [N_out, K]; column v = kd*9 + kh*3 + kw with kd on x,
 * kh on y, kw on z (conv3d_wgsl.ts:91-101,115-117); value = input row of the
 * neighbour with the same batch index, or -1 (absent / out of range).
 *
 * All pointers are caller-owned device pointers; the library never frees
 * caller memory.  Calls enqueue work on the handle's stream and return; no C++
 * exception crosses this boundary and nothing calls abort().  One handle per
 * host thread.
 */
#ifndef SPARSE_CONV_B200_H
#define SPARSE_CONV_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define SC_API __attribute__((visibility("default")))
#else
#define SC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum sc_status {
  SC_OK = 0,
  SC_EINVAL = 1,        /* bad argument (null pointer, size, alignment, shape) */
  SC_EDUP_COORD = 2,    /* two rows share (b, x, y, z) */
  SC_ERANGE = 3,        /* b outside [0, 32767] or x, y, z outside [0, 65535] */
  SC_ECUDA = 4,         /* CUDA runtime/driver error */
  SC_ENCCL = 5,         /* collective error (sharded calls) */
  SC_ETIMEOUT = 6,      /* a bounded device-side wait expired */
  SC_ENOMEM = 7,        /* device allocation failed */
  SC_EUNSUPPORTED = 8   /* valid request this build does not implement */
} sc_status;

typedef enum sc_dtype { SC_F32 = 0, SC_BF16 = 1, SC_F16 = 2 } sc_dtype;

/* neighbour-map construction modes */
enum { SC_MAP_HASH = 0, SC_MAP_SORT = 1 };
/* kernel-map kinds */
enum { SC_KMAP_SUBM = 0, SC_KMAP_DOWN2 = 1, SC_KMAP_UP2 = 2 };
/* build flags */
enum {
  SC_BUILD_NO_TILE_SORT = 1u, /* keep output order for tiles (no mask sort) */
  SC_BUILD_DEFER_CHECK = 2u,  /* do not wait for the device error word */
  SC_BUILD_HALO = 4u          /* submanifold maps: tiles in output order plus per-tile
                                 halo lists for the halo-staged conv (waits once to read
                                 the largest halo) */
};
/* conv epilogue flags, applied in this order: +bias, LayerNorm, SiLU, +residual */
enum { SC_EPI_SILU = 1u, SC_EPI_RESIDUAL = 2u, SC_EPI_LAYERNORM = 4u };

typedef struct sc_config {
  int32_t device;       /* CUDA device ordinal */
  int32_t map_mode;     /* SC_MAP_HASH (default) or SC_MAP_SORT */
  int32_t debug_bounds; /* nonzero: check every gathered row index on device */
  int32_t reserved;
} sc_config;

typedef struct sc_kmap_info {
  int32_t kind;          /* SC_KMAP_* */
  int32_t kernel_volume; /* K: 27 (3x3x3) or 8 (2x2x2) */
  int64_t n_in;          /* rows of the input features */
  int64_t n_out;         /* rows of the output */
  int64_t num_pairs;     /* M: valid (output, offset) pairs */
  int64_t num_tiles;     /* 128-row output tiles */
  int64_t tile_pairs;    /* sum over tiles of 128 * popcount(tile offset mask) */
  int64_t halo_max;      /* largest per-tile halo of an SC_BUILD_HALO map, else -1 */
} sc_kmap_info;

typedef struct sc_handle sc_handle;
typedef struct sc_kmap sc_kmap;

/* Library version string. */
SC_API const char* sc_version(void);

/* Fills `cfg` with defaults (device 0, hash map mode, no debug checks). */
SC_API void sc_config_default(sc_config* cfg);

/* Per-device handle: owns the stream binding, memory pool settings and the
 * last-error string.  Replaces the per-call GPUContext of the TS port
 * (src/runtime/device.ts:30). */
SC_API sc_status sc_create(sc_handle** out, const sc_config* cfg);
SC_API sc_status sc_destroy(sc_handle* h);
/* Enqueue all later work on `stream` (a cudaStream_t; NULL = legacy default). */
SC_API sc_status sc_set_stream(sc_handle* h, void* stream);

/* CTAs of the persistent tensor-core conv: 0 (default) = one per SM.  A
 * smaller grid leaves SMs free for a collective that runs beside the conv
 * (the halo exchange of a sharded conv).  No counterpart in the reference. */
SC_API sc_status sc_set_conv_ctas(sc_handle* h, int32_t max_ctas);
/* Waits for all work enqueued on the handle's stream, then returns (and
 * clears) the first error a kernel recorded in the handle's device error word
 * since the last call: SC_ETIMEOUT (a bounded device wait ran out) or
 * SC_EINVAL (sc_halo_push skipped a row with a bad destination). */
SC_API sc_status sc_synchronize(sc_handle* h);
/* Human-readable description of the last error on this handle. */
SC_API const char* sc_last_error(const sc_handle* h);
/* Number of CUDA kernels this handle has launched so far (instrumentation;
 * no counterpart in the reference). */
SC_API uint64_t sc_launch_count(const sc_handle* h);

/* Submanifold neighbour map for a 3x3x3 kernel with dilation `dilation`.
 * Replaces passes 0+1 (src/sparse/ops/conv3d.ts:73-151,
 * conv3d_wgsl.ts:44-128) and hashmap_fallback.py (README.md:111).
 * Unless SC_BUILD_DEFER_CHECK is set, waits for the build and returns
 * SC_EDUP_COORD / SC_ERANGE for bad coordinates. */
SC_API sc_status sc_kmap_build(sc_handle* h, const int32_t* coords, int64_t n, int32_t kernel_size, int32_t dilation,
                        uint32_t flags, sc_kmap** out);

/* As sc_kmap_build, but only the first n_out rows of `coords` are outputs;
 * neighbours are looked up among all n_in rows.  Used by sharded convs: a
 * rank's owned voxels come first, its halo voxels (neighbours owned by other
 * ranks) after them.  Replaces the same passes as sc_kmap_build. */
SC_API sc_status sc_kmap_build_ex(sc_handle* h, const int32_t* coords, int64_t n_in, int64_t n_out,
                                  int32_t kernel_size, int32_t dilation, uint32_t flags, sc_kmap** out);

/* As sc_kmap_build_ex, with outputs rows [out_begin, out_end) of `coords`
 * (map row j is output j = input row out_begin + j); neighbours are looked up
 * among all n_in rows.  A sharded conv orders a rank's owned voxels interior
 * first (no neighbour position owned by another rank), then boundary, then its
 * halo, and builds one map per output range so the interior conv can run
 * while the halo is in flight.  Replaces the same passes as sc_kmap_build. */
SC_API sc_status sc_kmap_build_range(sc_handle* h, const int32_t* coords, int64_t n_in, int64_t out_begin,
                                     int64_t out_end, int32_t kernel_size, int32_t dilation, uint32_t flags,
                                     sc_kmap** out);

/* As sc_kmap_build_range with a dilation per axis: offset v = kd*9 + kh*3 + kw
 * is ((kd-1)*dil_x, (kh-1)*dil_y, (kw-1)*dil_z), i.e. the reference's
 * (dilD, dilH, dilW) with kd on x, kh on y, kw on z
 * (src/sparse/ops/conv3d.ts:22,43-45; conv3d_wgsl.ts:91-101,115-117).  Each
 * dilation in [1, 1024].  Replaces the same passes as sc_kmap_build. */
SC_API sc_status sc_kmap_build_dilated(sc_handle* h, const int32_t* coords, int64_t n_in, int64_t out_begin,
                                       int64_t out_end, int32_t dil_x, int32_t dil_y, int32_t dil_z, uint32_t flags,
                                       sc_kmap** out);

/* Stride-2 2x2x2 down-sample map: parents are the unique (b, x>>1, y>>1, z>>1)
 * in ascending lexicographic order; map column = (x&1)*4 + (y&1)*2 + (z&1).
 * Replaces the stride-2 sparse conv of trellis2/modules/sparse/conv (absent
 * from the reference tree; semantics fixed by this ABI).  Waits for the
 * parent count. */
SC_API sc_status sc_kmap_build_down2(sc_handle* h, const int32_t* coords, int64_t n, uint32_t flags, sc_kmap** out);

/* Transposed 2x2x2 map from a down-sample map: outputs are the fine rows,
 * inputs the parents; row c uses column slot(c) and reads parent(c). */
SC_API sc_status sc_kmap_build_up2(sc_handle* h, const sc_kmap* down, uint32_t flags, sc_kmap** out);

/* Parent coords of a down-sample map: int32 [n_out, 4]. */
SC_API sc_status sc_kmap_out_coords(sc_handle* h, const sc_kmap* km, int32_t* coords_out);

/* Submanifold 3x3x3 neighbour map written straight into `map_out`
 * (int32 [n, 27], caller-owned device memory) without allocating any device
 * memory.  No counterpart in the reference.  For callers that must not let a
 * library allocate device memory (a host runtime that budgets all device
 * memory itself, or a latency-sensitive path that cannot wait on an allocator).
 * Scratch is a fixed 8 MiB __device__ array held by every GPU that loads the
 * library: n must be <= SC_NOALLOC_MAX_VOXELS (else SC_EINVAL).  Calls share
 * that scratch, so calls that overlap on the GPU race; order them.  The first
 * call on a device looks up the scratch address.  Every call waits for its
 * build on the handle's stream and returns its status, so it cannot be made
 * while that stream is being captured (SC_EINVAL, nothing enqueued). */
#define SC_NOALLOC_MAX_VOXELS 131072
SC_API sc_status sc_kmap_build_noalloc(sc_handle* h, const int32_t* coords, int64_t n, int32_t dilation,
                                       int32_t* map_out);

/* Map whose tiles are `first`'s followed by `second`'s: both submanifold maps
 * over the same input rows, typically two output ranges of one shard built
 * with sc_kmap_build_range (rows that read no halo row, then the rest).
 * Output j of `second` becomes output first.n_out + j.  The conv schedules
 * every tile of `second` after all tiles of `first`, and sc_conv3d_halo waits
 * for the halo exchange only before those.  Halo data of the parts is not
 * kept; the parts stay valid and may be freed.  `flags`: only
 * SC_BUILD_DEFER_CHECK applies (without it the call waits for the copy and
 * returns the parts' build status).  No counterpart in the reference (its
 * conv runs on one device). */
SC_API sc_status sc_kmap_concat(sc_handle* h, const sc_kmap* first, const sc_kmap* second, uint32_t flags,
                                sc_kmap** out);

/* Writes the canonical int32 [n_out, K] map (for bit-exact checks). */
SC_API sc_status sc_kmap_export(sc_handle* h, const sc_kmap* km, int32_t* map_out);

/* Sizes and pair counts (waits for the build to finish). */
SC_API sc_status sc_kmap_get_info(sc_handle* h, const sc_kmap* km, sc_kmap_info* info);

/* Waits for the build and returns its device-side status. */
SC_API sc_status sc_kmap_check(sc_handle* h, const sc_kmap* km);

SC_API sc_status sc_kmap_free(sc_handle* h, sc_kmap* km);

/* out[n] = epilogue(bias + sum_v W[:, v, :] . feats[map[n, v]]).
 * Replaces pass 2 (src/sparse/ops/conv3d.ts:154-221, conv3d_wgsl.ts:132-231)
 * and conv_none.py (README.md:109).  bf16/f16: tcgen05 tensor cores with f32
 * accumulation; f32: f32 FMA.  `residual` is [n_out, Co] (SC_EPI_RESIDUAL),
 * LayerNorm has no affine and uses `ln_eps`. */
SC_API sc_status sc_conv3d(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight, const void* bias,
                    const void* residual, void* out, int32_t ci, int32_t co, sc_dtype dtype, uint32_t epilogue,
                    float ln_eps);

/* Named entry points for the three operator kinds; each checks the map kind
 * and forwards to sc_conv3d. */
SC_API sc_status sc_conv3d_subm(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight, const void* bias,
                         const void* residual, void* out, int32_t ci, int32_t co, sc_dtype dtype, uint32_t epilogue,
                         float ln_eps);
SC_API sc_status sc_conv3d_down2(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight,
                          const void* bias, void* out, int32_t ci, int32_t co, sc_dtype dtype, uint32_t epilogue);
SC_API sc_status sc_conv3d_up2(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight, const void* bias,
                        void* out, int32_t ci, int32_t co, sc_dtype dtype, uint32_t epilogue);

/* Depthwise 3x3x3 submanifold conv: out[n, c] = bias[c] + sum_v W[c, v] *
 * feats[map[n, v], c], weight (C, 3, 3, 3, 1) with v = kd*9 + kh*3 + kw, f32
 * accumulation in ascending v.  This is the decoder ConvNeXt block's dw_conv
 * (src/models/sparse_unet_vae_decoder.ts:48-59,122-132, which runs it through
 * the dense conv of src/sparse/ops/conv3d.ts:40-75) for a depthwise
 * checkpoint weight.  `km` must be a 3x3x3 submanifold map; channels a
 * multiple of 8; feats and out 16-byte aligned device arrays [n_in, C] and
 * [n_out, C]; bias may be NULL. */
SC_API sc_status sc_conv3d_depthwise(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight,
                              const void* bias, void* out, int32_t channels, sc_dtype dtype);

/* 2x2x2 subdivision.  Every voxel (b, x, y, z) of coords [n, 4] becomes the
 * children (b, 2x+i, 2y+j, 2z+k), child s = i*4 + j*2 + k, written in
 * (voxel, s) order to out_coords [*, 4]; out_parent (may be NULL) receives the
 * voxel index of every child.  child_mask (n bytes, may be NULL = all 8)
 * keeps child s of voxel p when bit s of child_mask[p] is set.  With
 * out_feats, child rows get a copy of their parent's row of feats (row_bytes
 * per row, a multiple of 16; needs out_parent).  *n_out receives the number
 * of children; with out_coords NULL nothing is written (count only).  More
 * children than capacity rows gives SC_ERANGE with *n_out set.  With a mask
 * the call synchronizes the handle's stream to read the count.  Coordinates
 * must be in [0, 2^30).  This is the upsample that the TS decoder replaces by
 * a doubled spatialShape (src/models/sparse_unet_vae_decoder.ts:155-175). */
SC_API sc_status sc_subdivide2(sc_handle* h, const int32_t* coords, int64_t n, const uint8_t* child_mask,
                        const void* feats, int32_t row_bytes, int32_t* out_coords, int32_t* out_parent,
                        void* out_feats, int64_t capacity, int64_t* n_out);

/* Variable-length scaled dot-product attention (the SLat flow model's sparse
 * self / cross attention, src/sparse/ops/attention.ts:24-80 with the dense op
 * of src/dense/ops/attention.ts:2,61): for every sequence b and head h,
 * out[i, h] = softmax_j(scale * q[i, h] . k[j, h]) v[j, h] over the key rows j
 * of sequence b.  q / out are [cu_seqlens_q[batch], num_heads, head_dim],
 * k / v are [cu_seqlens_kv[batch], num_heads, head_dim] device arrays (16-byte
 * aligned); cu_seqlens_q / cu_seqlens_kv are HOST arrays of batch + 1
 * non-decreasing offsets starting at 0 (the reference passes Uint32Array
 * cuSeqlensQ / cuSeqlensKV).  head_dim must be 64; dtype bf16 or f16; f32
 * accumulation, P rounded to the input type for the second product.  Query
 * rows of a sequence with no key rows get zeros.  scale is usually
 * 1 / sqrt(head_dim). */
SC_API sc_status sc_attention_varlen(sc_handle* h, const void* q, const void* k, const void* v, void* out,
                              const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_kv, int32_t batch,
                              int32_t num_heads, int32_t head_dim, float scale, sc_dtype dtype);

/* Row LayerNorm (no affine) + optional SiLU, in place on [n, c] features
 * (src/dense/ops/layer_norm.ts:28-60, src/dense/ops/silu.ts:20-31). */
SC_API sc_status sc_layernorm_silu(sc_handle* h, void* x, int64_t n, int32_t c, sc_dtype dtype, int32_t apply_silu,
                            float eps);

/* ---- Halo exchange over peer memory (sharded convs on the GPUs of one node).
 * Replaces the NCCL all-to-all of the halo rows (the exchange step of a
 * Morton-sharded conv); no counterpart in the reference, whose conv runs on
 * one device.  Every rank allocates a peer buffer, shares its IPC handle
 * (SC_IPC_HANDLE_BYTES opaque bytes) with the other ranks and opens theirs. */
#define SC_IPC_HANDLE_BYTES 64

/* Device buffer of `bytes` (zeroed) that other processes can open; the
 * handle bytes go to `ipc_handle_out`. */
SC_API sc_status sc_peer_alloc(sc_handle* h, size_t bytes, void** ptr, void* ipc_handle_out);
SC_API sc_status sc_peer_free(sc_handle* h, void* ptr);
/* Maps another process's peer buffer into this device's address space. */
SC_API sc_status sc_peer_open(sc_handle* h, const void* ipc_handle, void** peer_ptr);
SC_API sc_status sc_peer_close(sc_handle* h, void* peer_ptr);

/* Copies rows to other ranks and signals them: row k of the send list is
 * `feats` row src_row[k] (row_bytes bytes, a multiple of 16), stored at byte
 * offset dst_off[k] of peer buffer dst_peer[k] (peer_bufs: device array of
 * `world` buffer addresses).  dst_off[k] must be a non-negative multiple of
 * 16 and dst_peer[k] in [0, world) and != rank; a row that breaks either rule
 * is not stored and records SC_EINVAL in the handle's device error word (see
 * sc_synchronize).  The caller keeps dst_off[k] + row_bytes within the
 * destination's buffer.  When every row has been stored, writes `epoch`
 * to word `rank` of each peer's flag array (peer_flags: device array of
 * `world` flag-array addresses).  2 <= world <= 32.  Enqueued on the
 * handle's stream. */
SC_API sc_status sc_halo_push(sc_handle* h, const void* feats, int32_t row_bytes, const int32_t* src_row,
                              const int32_t* dst_peer, const int64_t* dst_off, int64_t n_send,
                              void* const* peer_bufs, uint32_t* const* peer_flags, int32_t world, int32_t rank,
                              uint32_t epoch);

/* sc_conv3d on a submanifold map whose gathers read halo rows filled by
 * sc_halo_push of exchange `epoch`: the conv waits on the device until word r
 * of `flags` (4-byte aligned) is >= epoch for every r != rank, inside the
 * conv kernel before
 * its first tile from the second part of a concatenated map (before its first
 * tile for other maps), so tiles that read no halo row run while the exchange
 * is in flight.  The conv finishes only after the exchange has arrived.  A
 * wait longer than half a second records SC_ETIMEOUT (see sc_synchronize).
 * f32 convs and the halo-staged kernel wait in a separate launch first.
 * Replaces sc_halo_wait followed by sc_conv3d. */
SC_API sc_status sc_conv3d_halo(sc_handle* h, const sc_kmap* km, const void* feats, const void* weight,
                                const void* bias, const void* residual, void* out, int32_t ci, int32_t co,
                                sc_dtype dtype, uint32_t epilogue, float ln_eps, const uint32_t* flags,
                                int32_t world, int32_t rank, uint32_t epoch);

/* Waits on the device until word r of `flags` (this rank's flag array, 4-byte
 * aligned) is
 * >= epoch for every r != rank; a wait longer than one second records
 * SC_ETIMEOUT in the handle's device error word (see sc_synchronize) and
 * returns.  Enqueued on the handle's stream. */
SC_API sc_status sc_halo_wait(sc_handle* h, const uint32_t* flags, int32_t world, int32_t rank, uint32_t epoch);

#ifdef __cplusplus
}
#endif

#endif /* SPARSE_CONV_B200_H */
