/*
 * s3dsp — B200 (sm_100a) sparse-convolution library for the SAM 3D Objects
 * structured-latent path: coordinate hash, kernel maps, implicit-gather
 * GEMM convolutions and their fused epilogues.
 *
 * Drop-in boundary. In sam3d.cpp this path is reached through internal C++:
 *   - decode_object_mesh            src/objects_runtime/session.cpp:895-996
 *   - the SLat sampling loop        src/objects_runtime/session.cpp:1564-1763
 * which build host tables (src/objects_runtime/sparse_ops.hpp:11-78) and GGML
 * graphs (mesh_decoder_graph.cpp:42-132, slat_flow_graph.cpp:112-275) and run
 * them through Backend (backend.hpp:16-92). Each entry point below names the
 * reference piece it replaces.
 *
 * Conventions mirror the reference's public C API (include/sam3d.h:20-40):
 *   - every fallible call returns s3d_status and takes a caller-owned error
 *     buffer (error, error_capacity): success clears it, failure writes a
 *     truncated NUL-terminated message; NULL,0 discards diagnostics;
 *   - opaque handles with create/free; no exceptions, STL or struct layouts
 *     cross the ABI; plain pointers and sizes only;
 *   - device pointers passed in are caller-owned and must stay valid until the
 *     work queued on the context's stream has finished;
 *   - a context (and everything created from it) is not thread-safe; separate
 *     contexts may be used concurrently.
 * All work is queued on the context's CUDA stream. Unless stated otherwise a
 * call returns once the work is queued (stream order), not completed.
 */
#ifndef S3DSP_H
#define S3DSP_H

#include <stdint.h>

#define S3DSP_API __attribute__((visibility("default")))

#ifdef __cplusplus
extern "C" {
#endif

/* Same values as include/sam3d.h:22-26 in the reference. */
typedef uint32_t s3d_status;
#define S3D_OK UINT32_C(0)
#define S3D_INVALID_ARGUMENT UINT32_C(1)
#define S3D_OUT_OF_MEMORY UINT32_C(2)
#define S3D_INTERNAL_ERROR UINT32_C(3)

typedef struct s3dsp_context s3dsp_context;
typedef struct s3dsp_hash s3dsp_hash;
typedef struct s3dsp_kmap s3dsp_kmap;
typedef struct s3dsp_slat_tables s3dsp_slat_tables;
typedef struct s3dsp_fc_tables s3dsp_fc_tables;
typedef struct s3dsp_mesh s3dsp_mesh;
typedef struct s3dsp_gguf s3dsp_gguf;
typedef struct s3dsp_shard s3dsp_shard;

/* element types */
#define S3DSP_F32 UINT32_C(0)
#define S3DSP_BF16 UINT32_C(1)
#define S3DSP_F16 UINT32_C(2)

/* arithmetic of a convolution */
#define S3DSP_PREC_F32_STRICT UINT32_C(0) /* f32 FMA, f32 accumulation */
#define S3DSP_PREC_BF16 UINT32_C(1)       /* bf16 tcgen05 MMA, f32 accumulation in TMEM */
#define S3DSP_PREC_F32_3XTF32 UINT32_C(2) /* f32 in / out on the tensor cores: operands split into a TF32
                                             high part and its remainder, lo*hi + hi*lo + hi*hi
                                             tcgen05 MMAs (kind::tf32) into an f32 TMEM accumulator.
                                             s3dsp_conv only (no prologue, no CTA pairs) */

/* weight layouts accepted by s3dsp_weights_pack (all row-major as stored in GGUF) */
#define S3DSP_LAYOUT_SLAT_ROW UINT32_C(0)    /* (Cout, 27, Cin): scripts/objects/gguf_schema.py:326-334 */
#define S3DSP_LAYOUT_MESH_PACKED UINT32_C(1) /* (kvol, Cout, Cin): convert_sam3d_to_gguf.py:481-492 */
#define S3DSP_LAYOUT_LINEAR UINT32_C(2)      /* (Cout, Cin): gb_linear weights, graph_builder.cpp:44-54 */
#define S3DSP_LAYOUT_SPCONV_1X1 UINT32_C(3)  /* raw spconv (Cout,1,1,1,Cin) buffer read as (Cin, Cout),
                                                the 1x1 quirk of convert_sam3d_to_gguf.py:483-488 */
#define S3DSP_LAYOUT_TRANSPOSED_2X2X2 UINT32_C(4) /* (8, Cout, Cin): learned stride-2 subdivide, child
                                                     j = xb*4+yb*2+zb (no reference counterpart) */

/* dense neighbour-table export formats */
#define S3DSP_SENTINEL_SLAT_N UINT32_C(0)   /* missing -> n (zero row), sparse_ops.hpp:24-29 */
#define S3DSP_SENTINEL_MESH_NEG1 UINT32_C(1) /* missing -> -1, sparse_ops.cpp:367 */

/* conv epilogue / prologue flags */
#define S3DSP_EPI_SILU UINT32_C(1)      /* apply SiLU after bias (and residual) */
#define S3DSP_PRO_AFFINE_SILU UINT32_C(2) /* gathered x -> silu((x - sub[c]) * mul[c] + add[c]) */
#define S3DSP_EPI_GELU UINT32_C(64)     /* apply GELU, tanh form 0.5x(1 + tanh(sqrt(2/pi)(x + 0.044715x^3))),
                                           after bias (and residual); the MLP of gs_decoder_graph.cpp:140 */
#define S3DSP_CONV_TILE128 UINT32_C(8)   /* BF16: force one CTA per 128-row tile */
#define S3DSP_CONV_STREAM_K UINT32_C(16) /* BF16: force 256-row tiles split evenly over all SMs
                                          (stream-K). No kernel flag: chosen by size, see s3dsp_conv_kernel */
#define S3DSP_CONV_STREAM_K128 UINT32_C(32) /* BF16: force 128-row tiles split evenly over all SMs */
#define S3DSP_CONV_SPLIT_PAIRS UINT32_C(128) /* BF16: force 256-row tiles, each on a CTA pair (a cluster of
                                            2) that splits the kernel offsets and adds its two partial
                                            sums in distributed shared memory */
#define S3DSP_CONV_CTA_PAIR UINT32_C(4)  /* BF16: tcgen05 CTA pairs (256-row MMA over two tiles) instead of
                                          one CTA per 128-row tile; same results, slower on B200 today */
#define S3DSP_CONV_HALO UINT32_C(256)    /* BF16: force the per-tile input halo kernel (one source, cin <= 256,
                                            cout <= 128, kvol <= 27; other layers ignore the flag) */

/* context flags */
#define S3DSP_CONTEXT_DEFERRED_CHECKS UINT32_C(1) /* device-detected input errors are reported by
                                                     s3dsp_context_check instead of at each call */
#define S3DSP_CONTEXT_OWN_STREAM UINT32_C(2)      /* create (and own) a new non-blocking stream */
#define S3DSP_CONTEXT_COPY_STREAMS UINT32_C(4)    /* the context also owns a copy-in and a copy-out
                                                     stream for its host-buffer calls (see
                                                     s3dsp_context_fork / s3dsp_context_join) */

S3DSP_API uint32_t s3dsp_abi_version(void);

/* ---------------------------------------------------------------------------
 * Context: one CUDA device + one stream (replaces the per-stage Backend,
 * backend.cpp:44-118). `stream` is a cudaStream_t; NULL is the legacy default
 * stream, as everywhere in CUDA. With S3DSP_CONTEXT_OWN_STREAM the context
 * creates its own non-blocking stream instead and `stream` is ignored.
 * ------------------------------------------------------------------------- */
S3DSP_API s3d_status s3dsp_context_create(int32_t device, void *stream, uint32_t flags,
                                          s3dsp_context **out, char *error,
                                          uint64_t error_capacity);
S3DSP_API void s3dsp_context_free(s3dsp_context *ctx);
S3DSP_API void *s3dsp_context_stream(const s3dsp_context *ctx);
/* Size this context's persistent and SM-proportional grids (the stream-K
 * conv, the streaming kernels) for `sms` SMs instead of all of the device's,
 * so that work on another stream -- a halo exchange's NCCL kernel beside an
 * interior conv, say -- finds SMs free. 0 restores the device's count. The
 * kernel choice of s3dsp_conv follows the same count. No counterpart in the
 * reference (one stream per Backend). */
S3DSP_API s3d_status s3dsp_context_set_sm_limit(s3dsp_context *ctx, int32_t sms, char *error,
                                                uint64_t error_capacity);
/* Waits for the stream (and, with S3DSP_CONTEXT_COPY_STREAMS, the copy
 * streams) and reports (then clears) any device-detected input error
 * recorded since the last check. */
S3DSP_API s3d_status s3dsp_context_check(s3dsp_context *ctx, char *error, uint64_t error_capacity);
/* Copy streams (S3DSP_CONTEXT_COPY_STREAMS). Such a context runs the
 * host-buffer entry points (s3dsp_res_block_gn_host and its queued form) over
 * three streams: the host -> device copies on its copy-in stream, the tables
 * and kernels on its stream, the device -> host copy on its copy-out stream,
 * through a ring of three staging slots that the context keeps (device
 * memory from the library pool, sized by the largest call so far, freed with
 * the context). Successive queued calls then overlap one call's upload, the
 * next one's kernels and the previous one's download; on PCIe the two copy
 * directions run at the same time. s3dsp_context_fork orders the copy
 * streams after everything queued on the context's stream so far (call it
 * before queued calls whose host inputs earlier stream work produces);
 * s3dsp_context_join orders the context's stream after everything queued on
 * the copy streams so far (an event recorded on the stream after a join, or
 * s3dsp_context_check, then covers every queued call's read-back). Without
 * the flag both return S3D_OK and do nothing. No counterpart in the
 * reference (its Backend::run copies and computes on one queue,
 * backend.hpp:16-92). */
S3DSP_API s3d_status s3dsp_context_fork(s3dsp_context *ctx, char *error, uint64_t error_capacity);
S3DSP_API s3d_status s3dsp_context_join(s3dsp_context *ctx, char *error, uint64_t error_capacity);

/* Device buffers for a host that links only this library (the counterpart of
 * the reference's Backend::alloc / set_input_f32 / set_input_i32 /
 * get_tensor_f32, backend.hpp:16-92): s3dsp_device_alloc returns `bytes` of
 * device memory on the context's device (cudaMalloc; freed by
 * s3dsp_device_free, which first waits for the context's stream);
 * s3dsp_copy_to_device queues a host -> device copy on the context's stream
 * (the host buffer must stay valid until the stream reaches it: pageable
 * memory is staged before the call returns); s3dsp_copy_to_host copies
 * device -> host and waits for it (synchronous). */
S3DSP_API s3d_status s3dsp_device_alloc(s3dsp_context *ctx, uint64_t bytes, void **out, char *error,
                                        uint64_t error_capacity);
S3DSP_API void s3dsp_device_free(s3dsp_context *ctx, void *d_ptr);
S3DSP_API s3d_status s3dsp_copy_to_device(s3dsp_context *ctx, void *d_dst, const void *h_src, uint64_t bytes,
                                          char *error, uint64_t error_capacity);
S3DSP_API s3d_status s3dsp_copy_to_host(s3dsp_context *ctx, void *h_dst, const void *d_src, uint64_t bytes,
                                        char *error, uint64_t error_capacity);

/* Device memory the library holds on `device`. Every table, map and scratch
 * buffer the library allocates comes from its own stream-ordered pool (made
 * by the first s3dsp_context_create on the device; memory freed by the
 * library stays in that pool for reuse). The device's default pool, which
 * the host process may use, is left as it was. Reports the pool's reserved
 * bytes, bytes in use and the high-water mark of bytes in use (any pointer
 * may be NULL); reset_high != 0 then resets that mark to the current use.
 * The reference reserves graph memory through GGML's allocator per stage
 * (backend.cpp:44-118); this is the counterpart for accounting. */
S3DSP_API s3d_status s3dsp_memory_stats(int32_t device, uint64_t *reserved, uint64_t *used,
                                        uint64_t *used_high, int32_t reset_high, char *error,
                                        uint64_t error_capacity);

/* ---------------------------------------------------------------------------
 * Coordinate hash. Replaces the std::map / unordered_map indexes of
 * SlatTables::build (sparse_ops.cpp:119-124) and MeshSubdivideTables::build
 * (sparse_ops.cpp:299-333; FNV key hash :32-45).
 * d_coords: device int32 [n, 4] rows (batch, x, y, z); the hash keeps its own
 * copy. Domain: 0 <= batch < 32768 and -32768 <= x, y, z < 32768. Duplicate
 * coordinates keep the first row (the reference's std::map emplace rule);
 * `reject_duplicates` makes them an error instead (MeshSubdivideTables,
 * sparse_ops.cpp:325-333). Synchronous check unless DEFERRED_CHECKS.
 * ------------------------------------------------------------------------- */
S3DSP_API s3d_status s3dsp_hash_build(s3dsp_context *ctx, const int32_t *d_coords, int64_t n,
                                      int32_t reject_duplicates, s3dsp_hash **out, char *error,
                                      uint64_t error_capacity);
S3DSP_API void s3dsp_hash_free(s3dsp_context *ctx, s3dsp_hash *hash);
S3DSP_API int64_t s3dsp_hash_size(const s3dsp_hash *hash);
/* d_rows[i] = first row whose coords equal d_query[i], or -1. */
S3DSP_API s3d_status s3dsp_hash_lookup(s3dsp_context *ctx, const s3dsp_hash *hash,
                                       const int32_t *d_query, int64_t m, int32_t *d_rows,
                                       char *error, uint64_t error_capacity);

/* ---------------------------------------------------------------------------
 * The coordinate pipeline in front of the path (src/objects_runtime/
 * session.cpp). Each call returns the row count in *count (host) and so
 * synchronises the context's stream; rows are written only when the count
 * fits `capacity` (else S3D_INVALID_ARGUMENT, *count still set). Input order
 * is kept. Coordinates must lie in the hash domain (0 <= b < 32768,
 * |x|,|y|,|z| < 32768).
 * ------------------------------------------------------------------------- */
/* SS occupancy argwhere (session.cpp:1436-1441): d_occ is a C-order f32
 * [nx, ny, nz] grid; every cell > 0 gives a row (batch, x, y, z), x-major. */
S3DSP_API s3d_status s3dsp_occupancy_coords(s3dsp_context *ctx, const float *d_occ, int32_t nx,
                                            int32_t ny, int32_t nz, int32_t batch, int32_t *d_coords,
                                            int64_t capacity, int64_t *count, char *error,
                                            uint64_t error_capacity);
/* prune_surface_coords (session.cpp:129-166): keep the rows with some cell of
 * their (2*max_axis_dist+1)^3 neighbourhood unoccupied. */
S3DSP_API s3d_status s3dsp_prune_surface(s3dsp_context *ctx, const int32_t *d_coords, int64_t n,
                                         int32_t max_axis_dist, int32_t *d_out, int64_t capacity,
                                         int64_t *count, char *error, uint64_t error_capacity);
/* downsample_coords (session.cpp:168-236): n <= max_coords rows are copied
 * unchanged; otherwise every axis is rescaled by 1/factor about the box
 * centre (double arithmetic, round half up, clamped), first occurrences kept,
 * and above max_coords again max_coords rows are drawn by std::shuffle with
 * std::mt19937(seed) (on the host). */
S3DSP_API s3d_status s3dsp_downsample_coords(s3dsp_context *ctx, const int32_t *d_coords, int64_t n,
                                             int64_t max_coords, int32_t factor, uint32_t seed,
                                             int32_t *d_out, int64_t capacity, int64_t *count,
                                             char *error, uint64_t error_capacity);

/* ---------------------------------------------------------------------------
 * GS decoder Swin window tables and position embedding (GsTables::build,
 * src/objects_runtime/sparse_ops.cpp:182-270).
 * ------------------------------------------------------------------------- */
/* Windows of side `window` (8 in the reference) over the coordinates shifted
 * by `shift` (0 or 4): a window's id is the order of its first token; tokens
 * are grouped by window (table order inside) and windows laid out by token
 * count ascending (id order inside a count). d_bkt_idx[row] = token,
 * d_bwd_idx[token] = row (device, [n] each); h_buckets[3k..3k+2] = {tokens per
 * window, first row, windows} per distinct count (host). Synchronises the
 * context's stream; *n_buckets is set even when it exceeds bucket_capacity
 * (then S3D_INVALID_ARGUMENT). */
S3DSP_API s3d_status s3dsp_gs_window_tables(s3dsp_context *ctx, const int32_t *d_coords, int64_t n,
                                            int32_t shift, int32_t window, int32_t *d_bkt_idx,
                                            int32_t *d_bwd_idx, int32_t *h_buckets,
                                            int64_t bucket_capacity, int64_t *n_buckets, char *error,
                                            uint64_t error_capacity);
/* AbsolutePositionEmbedder: d_out [n, channels] f32, per axis channels/6 sines
 * then channels/6 cosines of coordinate * 10000^(-i/(channels/6)). */
S3DSP_API s3d_status s3dsp_ape(s3dsp_context *ctx, const int32_t *d_coords, int64_t n, int32_t channels,
                               float *d_out, char *error, uint64_t error_capacity);

/* ---------------------------------------------------------------------------
 * One volume over several GPUs (one process per GPU; no reference
 * counterpart: the reference runs one object on one device). Morton-ordered
 * slabs of (nearly) equal voxel count; each rank's own rows interior first
 * (no 26-neighbour on another rank), then boundary; ghost rows = other ranks'
 * voxels adjacent to the rank, grouped by owner, Morton order within; send
 * lists in the matching order. The plan is computed on the host from the
 * global coordinate list, identically on every rank, without communication.
 * ------------------------------------------------------------------------- */
S3DSP_API s3d_status s3dsp_shard_plan_morton(const int32_t *h_coords, int64_t n, int32_t world,
                                             int32_t rank, s3dsp_shard **out, char *error,
                                             uint64_t error_capacity);
S3DSP_API s3d_status s3dsp_shard_info(const s3dsp_shard *plan, int64_t *n_own, int64_t *n_interior,
                                      int64_t *n_ghost, int64_t *n_send);
/* host copies: own / ghost global row ids, per-peer recv / send counts
 * [world], send rows (indices into the own rows, grouped by destination);
 * any pointer may be NULL */
S3DSP_API s3d_status s3dsp_shard_lists(const s3dsp_shard *plan, int64_t *h_own, int64_t *h_ghost,
                                       int64_t *h_recv_counts, int64_t *h_send_counts,
                                       int64_t *h_send_rows);
S3DSP_API void s3dsp_shard_free(s3dsp_context *ctx, s3dsp_shard *plan);
/* NCCL is bound at run time (an already loaded libnccl.so.2, else the
 * system one); communicators passed to s3dsp_halo_exchange must come from
 * that NCCL, e.g. from s3dsp_nccl_comm_create with an id (128 bytes) made by
 * one rank with s3dsp_nccl_unique_id and shared by the host. */
S3DSP_API s3d_status s3dsp_nccl_unique_id(uint8_t *id, char *error, uint64_t error_capacity);
S3DSP_API s3d_status s3dsp_nccl_comm_create(s3dsp_context *ctx, int32_t world, int32_t rank,
                                            const uint8_t *id, void **comm, char *error,
                                            uint64_t error_capacity);
S3DSP_API void s3dsp_nccl_comm_free(void *comm);
/* Fills the ghost rows [n_own, n_own + n_ghost) of d_x ([n_own + n_ghost, c]
 * of dtype, device) with the peers' rows: the send rows are gathered, then
 * one NCCL group of send / recv per peer on the context's stream. */
S3DSP_API s3d_status s3dsp_halo_exchange(s3dsp_context *ctx, s3dsp_shard *plan, void *comm, void *d_x,
                                         int64_t c, uint32_t dtype, char *error,
                                         uint64_t error_capacity);

/* ---------------------------------------------------------------------------
 * On-disk formats. GGUF weight files (GGUFModel::load / get / u32 / i32 / f32
 * / str / str_array / i32_array, src/objects_runtime/gguf_loader.hpp:14-46):
 * header, metadata and tensor directory parsed on the host at open, tensor
 * bytes read on demand. SAMT raw tensors (save_raw_tensor / load_raw_tensor,
 * src/objects_runtime/common.hpp:34-48, common.cpp:59-119). ggml type ids:
 * F32 0, F16 1, Q4_0 2, Q4_1 3, Q8_0 8, Q4_K 12, I32 26, BF16 30.
 * ------------------------------------------------------------------------- */
S3DSP_API s3d_status s3dsp_gguf_open(const char *path, s3dsp_gguf **out, char *error,
                                     uint64_t error_capacity);
S3DSP_API void s3dsp_gguf_close(s3dsp_gguf *gguf);
S3DSP_API int64_t s3dsp_gguf_n_tensors(const s3dsp_gguf *gguf);
/* index of a tensor by name, -1 when absent (GGUFModel::get / has) */
S3DSP_API int64_t s3dsp_gguf_find(const s3dsp_gguf *gguf, const char *name);
/* ne[4] in ggml order (ne[0] fastest); nbytes of the stored data */
S3DSP_API s3d_status s3dsp_gguf_tensor_info(const s3dsp_gguf *gguf, int64_t index, const char **name,
                                            int32_t *ggml_type, int32_t *n_dims, int64_t *ne,
                                            uint64_t *nbytes);
/* metadata with defaults, GGUFModel semantics: u32/i32 accept the 32- and
 * 64-bit integer types; str / str_array copy a NUL-terminated string and
 * return its length (-1 when missing or of another type); i32_array and
 * array_len return the element count (-1 likewise). */
S3DSP_API uint32_t s3dsp_gguf_u32(const s3dsp_gguf *gguf, const char *key, uint32_t def);
S3DSP_API int32_t s3dsp_gguf_i32(const s3dsp_gguf *gguf, const char *key, int32_t def);
S3DSP_API float s3dsp_gguf_f32(const s3dsp_gguf *gguf, const char *key, float def);
S3DSP_API int64_t s3dsp_gguf_str(const s3dsp_gguf *gguf, const char *key, char *buf, uint64_t cap);
S3DSP_API int64_t s3dsp_gguf_array_len(const s3dsp_gguf *gguf, const char *key);
S3DSP_API int64_t s3dsp_gguf_str_array(const s3dsp_gguf *gguf, const char *key, int64_t i, char *buf,
                                       uint64_t cap);
S3DSP_API int64_t s3dsp_gguf_i32_array(const s3dsp_gguf *gguf, const char *key, int32_t *out,
                                       int64_t cap);
/* raw stored bytes of a tensor into host memory */
S3DSP_API s3d_status s3dsp_gguf_read(const s3dsp_gguf *gguf, int64_t index, void *h_dst,
                                     uint64_t capacity, char *error, uint64_t error_capacity);
/* a float tensor (F32, F16, BF16, Q8_0, Q4_0, Q4_1, Q4_K) to the device as
 * dtype (S3DSP_F32 or S3DSP_BF16), dequantised with GGML's block formulas;
 * synchronises the context's stream. */
S3DSP_API s3d_status s3dsp_gguf_load(s3dsp_context *ctx, const s3dsp_gguf *gguf, int64_t index,
                                     uint32_t dtype, void *d_out, int64_t capacity, char *error,
                                     uint64_t error_capacity);
/* a conv / linear weight by name straight into s3dsp_weights_pack's device
 * layout, after checking the stored shape: MESH_PACKED ne = {cout*cin,
 * kvol} (1x1 skips included, already transposed by the converter), SLAT_ROW
 * ne = {27*cin, cout}, LINEAR ne = {cin, cout}. */
S3DSP_API s3d_status s3dsp_gguf_load_weights(s3dsp_context *ctx, const s3dsp_gguf *gguf,
                                             const char *name, uint32_t layout, int32_t kvol,
                                             int64_t cin, int64_t cout, uint32_t precision,
                                             void *d_dst, char *error, uint64_t error_capacity);
/* device-to-device dequantisation of n elements stored as ggml_type */
S3DSP_API s3d_status s3dsp_dequantize(s3dsp_context *ctx, int32_t ggml_type, const void *d_src,
                                      int64_t n, uint32_t dtype, void *d_out, char *error,
                                      uint64_t error_capacity);
/* SAMT: "SAMT" | int32 ndims (1..8) | int64 ne[ndims] | int32 ggml type |
 * data; type 30 reads as I32 (26), as the reference's reader normalises it. */
S3DSP_API s3d_status s3dsp_samt_info(const char *path, int32_t *n_dims, int64_t *ne, int32_t *ggml_type,
                                     uint64_t *nbytes, char *error, uint64_t error_capacity);
S3DSP_API s3d_status s3dsp_samt_read(const char *path, void *h_dst, uint64_t capacity, char *error,
                                     uint64_t error_capacity);
S3DSP_API s3d_status s3dsp_samt_write(const char *path, int32_t n_dims, const int64_t *ne,
                                      int32_t ggml_type, const void *data, uint64_t nbytes,
                                      char *error, uint64_t error_capacity);

/* ---------------------------------------------------------------------------
 * GS decoder torso (gs_decoder_graph.cpp:13-155): its Linears are s3dsp_conv
 * with kmap NULL (S3DSP_EPI_GELU for the MLP, `residual` for the skips), its
 * norms s3dsp_layer_norm; these two calls are the rest.
 * ------------------------------------------------------------------------- */
/* y[i] = x[rows[i]] for i < n_out (x [n_in, c] of x_dtype, y [n_out, c] of
 * y_dtype): ggml_get_rows with the window tables' bucket order (:64). A row
 * index outside [0, n_in) gives a zero row and is reported by the next
 * status check. */
S3DSP_API s3d_status s3dsp_gather_rows(s3dsp_context *ctx, const void *x, uint32_t x_dtype, int64_t n_in,
                                       int64_t c, const int32_t *d_rows, int64_t n_out, void *y,
                                       uint32_t y_dtype, char *error, uint64_t error_capacity);
/* Swin window attention (:88-121). qkv f32 [n, 3c], rows in bucket order,
 * each row q | k | v with head h at columns h*d .. h*d+d-1 (d = c / heads:
 * 32 or 64). d_windows int32 [n_windows, 2] = (first row, rows) of each
 * window (the buckets' windows, consecutive rows). For every head and
 * window: softmax(q k^T / sqrt(d)) v over the window's rows, in f32 (max,
 * exp, sum, weighted values, as ggml_soft_max + ggml_mul_mat). Row i of the
 * result goes to out[d_scatter[i]] (the bucket order back to token order,
 * get_rows by bwd_idx), or out[i] when d_scatter is NULL. out f32 [n, c]. */
S3DSP_API s3d_status s3dsp_window_attention(s3dsp_context *ctx, const float *qkv, int64_t n, int64_t c,
                                            int32_t heads, const int32_t *d_windows, int64_t n_windows,
                                            const int32_t *d_scatter, float *out, char *error,
                                            uint64_t error_capacity);

/* ---------------------------------------------------------------------------
 * FlexiCubes extraction at resolution 256 (extract_object_mesh,
 * src/objects_runtime/mesh_extractor.cpp:95-377: SparseFeatures2Mesh followed
 * by inference-mode FlexiCubes), on the device.
 * ------------------------------------------------------------------------- */
/* Copies the dual-marching-cubes tables to the device: dmc [256][4][7] (edge
 * lists of each case's dual vertices, -1 padded), num_dual [256], check
 * [256][5] ({ambiguous, dx, dy, dz, replacement case}) -- the arrays of the
 * reference's generated src/objects_runtime/flexicubes_tables.hpp. */
S3DSP_API s3d_status s3dsp_flexicubes_tables_create(s3dsp_context *ctx, const int8_t *h_dmc,
                                                    const int8_t *h_num_dual, const int16_t *h_check,
                                                    s3dsp_fc_tables **out, char *error,
                                                    uint64_t error_capacity);
S3DSP_API void s3dsp_flexicubes_tables_free(s3dsp_context *ctx, s3dsp_fc_tables *tables);
/* d_raw [n, 101] f32 (row-major, channels: 0-7 corner SDF, 8-31 corner
 * deformation, 32-52 FlexiCubes weights, 53-100 corner colours), d_coords
 * [n, 4] int32 (batch 0, x, y, z in [0, 256)). Errors as the reference: batch
 * != 0, coordinate outside [0, 256), duplicate coordinate (the first bad row
 * decides the message). Synchronises the context's stream twice. The mesh
 * owns its device outputs: dual vertices [V, 3], their six attributes [V, 6],
 * triangles [F, 3] and the surface cubes (dense ids, x-major), their resolved
 * case ids and the surface edges [E, 2] (dense vertex ids). */
S3DSP_API s3d_status s3dsp_flexicubes_extract(s3dsp_context *ctx, const s3dsp_fc_tables *tables,
                                              const float *d_raw, const int32_t *d_coords, int64_t n,
                                              s3dsp_mesh **out, char *error, uint64_t error_capacity);
/* Counts of a mesh; any pointer may be NULL. */
S3DSP_API s3d_status s3dsp_mesh_info(const s3dsp_mesh *mesh, int64_t *n_vertices, int64_t *n_faces,
                                     int64_t *n_surface, int64_t *n_edges);
/* Device pointers owned by the mesh (valid until s3dsp_mesh_free); any output
 * pointer may be NULL. */
S3DSP_API s3d_status s3dsp_mesh_device(const s3dsp_mesh *mesh, const float **vertices,
                                       const float **attributes, const int32_t **faces,
                                       const int32_t **surface, const int32_t **cases,
                                       const int32_t **edges);
/* Copies the mesh to host memory (ObjectMesh + the topology taps) and
 * synchronises; any pointer may be NULL. */
S3DSP_API s3d_status s3dsp_mesh_copy(s3dsp_context *ctx, const s3dsp_mesh *mesh, float *h_vertices,
                                     float *h_attributes, int32_t *h_faces, int32_t *h_surface,
                                     int32_t *h_cases, int32_t *h_edges, char *error,
                                     uint64_t error_capacity);
S3DSP_API void s3dsp_mesh_free(s3dsp_context *ctx, s3dsp_mesh *mesh);

/* ---------------------------------------------------------------------------
 * Kernel maps. A kmap holds, per kernel offset o (o = kd*9 + kh*3 + kw with
 * (dx,dy,dz) = (kd-1, kh-1, kw-1), sparse_ops.cpp:132), the input row feeding
 * every output row (offset-major [kvol][n_out], -1 = none) plus a per-tile
 * bitmask of offsets that have any neighbour.
 * ------------------------------------------------------------------------- */
/* Submanifold 3x3x3 map of a coordinate set onto itself: SlatTables
 * conv_fine / conv_coarse (sparse_ops.cpp:126-142). Rows that duplicate an
 * earlier row's coordinates get no neighbours (reference behaviour). */
S3DSP_API s3d_status s3dsp_kmap_build_subm3(s3dsp_context *ctx, const s3dsp_hash *hash,
                                            s3dsp_kmap **out, char *error,
                                            uint64_t error_capacity);
/* The same map for the hash's first n_out rows only, gathering from all of
 * its rows (inputs: the n rows of the hash). Used by a volume split across
 * GPUs: a shard's own voxels come first, its halo (ghost) voxels after them.
 * No reference counterpart. */
S3DSP_API s3d_status s3dsp_kmap_build_subm3_rows(s3dsp_context *ctx, const s3dsp_hash *hash,
                                                 int64_t n_out, s3dsp_kmap **out, char *error,
                                                 uint64_t error_capacity);
/* The same for hash rows [row_begin, row_end): output row r of the map is hash
 * row row_begin + r (a shard's interior and boundary rows as two maps, so the
 * interior can be convolved while the halo is in flight). No reference
 * counterpart. */
S3DSP_API s3d_status s3dsp_kmap_build_subm3_range(s3dsp_context *ctx, const s3dsp_hash *hash,
                                                  int64_t row_begin, int64_t row_end, s3dsp_kmap **out,
                                                  char *error, uint64_t error_capacity);
/* Stride-2 subdivide of a parent set: MeshSubdivideTables::build
 * (sparse_ops.cpp:272-404). Writes the 8*n child coords (child row =
 * parent*8 + xb*4 + yb*2 + zb, coords 2p + bits) to d_child_coords [8n, 4]
 * and returns the child submanifold map. `parents` must be built with
 * reject_duplicates. */
S3DSP_API s3d_status s3dsp_subdivide(s3dsp_context *ctx, const s3dsp_hash *parents,
                                     int32_t *d_child_coords, s3dsp_kmap **out_child_kmap,
                                     char *error, uint64_t error_capacity);
S3DSP_API void s3dsp_kmap_free(s3dsp_context *ctx, s3dsp_kmap *kmap);
S3DSP_API int64_t s3dsp_kmap_rows(const s3dsp_kmap *kmap);
/* Dense row-major [n_out, 27] table in the reference's format (bit-exact with
 * SlatTables::conv_fine for SLAT_N, MeshSubdivideTables::neighbors for
 * MESH_NEG1). d_out is a device buffer of n_out*27 int32. */
S3DSP_API s3d_status s3dsp_kmap_export_dense(s3dsp_context *ctx, const s3dsp_kmap *kmap,
                                             uint32_t sentinel_mode, int32_t *d_out, char *error,
                                             uint64_t error_capacity);
/* A new map reading through a row table: entry (o, r) = d_rows[kmap(o, r)]
 * (none stays none). d_rows int32 [kmap input rows], values in
 * [0, n_rows_in); an out-of-range value becomes "none" and is reported by the
 * next status check. Used to gather coarse rows for a fine map (nearest
 * upsampling without building the upsampled rows). No reference counterpart:
 * the reference materialises the upsampled tensor (slat_flow_graph.cpp:185-190). */
S3DSP_API s3d_status s3dsp_kmap_compose(s3dsp_context *ctx, const s3dsp_kmap *kmap, const int32_t *d_rows,
                                        int64_t n_rows_in, s3dsp_kmap **out, char *error,
                                        uint64_t error_capacity);
/* Offset-sorted (in, out) pair lists: for each offset o in order, the pairs
 * with a neighbour, sorted by output row. d_in/d_out hold capacity int32
 * each (27*n_out always suffices); h_offsets receives kvol+1 host int64
 * start offsets. Synchronous: the call waits for the context's stream, so the
 * lists are complete when it returns. */
S3DSP_API s3d_status s3dsp_kmap_pairs(s3dsp_context *ctx, const s3dsp_kmap *kmap, int32_t *d_in,
                                      int32_t *d_out, int64_t capacity, int64_t *h_offsets,
                                      char *error, uint64_t error_capacity);

/* Allocation-free variant of s3dsp_kmap_pairs, for callers that may not
 * allocate device memory once they are running: a host whose memory is a
 * fixed, pre-reserved pool, or code that runs where cudaMalloc is not
 * allowed. It has no counterpart in the reference (whose tables are built on
 * the host). Same arguments and results as s3dsp_kmap_pairs; its scratch is a
 * static device array in the library, so the map may have at most 2^21
 * (2,097,152) output rows — larger maps fail with S3D_INVALID_ARGUMENT.
 * The kernel map may have at most 27 offsets. Every call looks up that
 * array's device address (cudaGetSymbolAddress); make the first call on a
 * device before any stream capture. All calls on a device share the array:
 * calls whose GPU work overlaps (different streams, concurrent contexts)
 * race and must be ordered by the caller. Synchronous, like s3dsp_kmap_pairs:
 * the call waits for its last kernel on the context's stream, so two calls
 * the host has ordered never overlap on the GPU. */
S3DSP_API s3d_status s3dsp_kmap_pairs_noalloc(s3dsp_context *ctx, const s3dsp_kmap *kmap,
                                              int32_t *d_in, int32_t *d_out, int64_t capacity,
                                              int64_t *h_offsets, char *error,
                                              uint64_t error_capacity);

/* ---------------------------------------------------------------------------
 * Weights. Converts a GGUF-layout weight (host or device `src`, f32/f16/bf16)
 * into the device layout a conv of `precision` consumes, at d_dst (size from
 * s3dsp_weights_packed_bytes). kvol = 27 (subm), 8 (transposed 2x2x2) or 1.
 * Replaces the load-time as_f32 casts (mesh_decoder_graph.cpp:10-12,
 * slat_flow_graph.cpp:14-41).
 * ------------------------------------------------------------------------- */
S3DSP_API int64_t s3dsp_weights_packed_bytes(uint32_t precision, int32_t kvol, int64_t cin,
                                             int64_t cout);
S3DSP_API s3d_status s3dsp_weights_pack(s3dsp_context *ctx, const void *src, uint32_t src_dtype,
                                        int32_t src_on_host, uint32_t layout, int32_t kvol,
                                        int64_t cin, int64_t cout, uint32_t precision,
                                        void *d_dst, char *error, uint64_t error_capacity);

/* ---------------------------------------------------------------------------
 * Sparse convolution (implicit gather GEMM, no atomics on outputs):
 *   out[r] = epi( sum_o W_o * pro(in[nbr_o(r) >> in_shift]) + bias
 *                 + residual[r >> res_shift] )
 * kmap == NULL means the identity map with kvol 1 (a Linear / 1x1 conv,
 * gb_linear graph_builder.cpp:44-54, or the mesh skip mesh_decoder_graph.cpp:
 * 126-129 with in_shift 3). Replaces the conv lambda of slat_flow_graph.cpp:
 * 112-155 and the convolution lambda of mesh_decoder_graph.cpp:81-103;
 * in_shift = 3 fuses repeat_children (:32-38).
 *   in:        [n_in, cin] of in_dtype (BF16 precision needs BF16 input)
 *   weight:    packed by s3dsp_weights_pack for `precision`
 *   bias:      f32 [cout] or NULL
 *   residual:  [*, cout] of res_dtype or NULL
 *   out:       [n_out, cout] of out_dtype
 *   pro_sub/pro_mul/pro_add: f32 [cin] when flags has PRO_AFFINE_SILU
 *   gn_partials: NULL, or f64 [s3dsp_gn_partials_count(n_out, cout, groups)]
 *              receiving per-tile GroupNorm sums of the output (pre-SiLU)
 * ------------------------------------------------------------------------- */
S3DSP_API int64_t s3dsp_gn_partials_count(int64_t n_rows, int64_t channels, int32_t groups);
S3DSP_API s3d_status s3dsp_conv(s3dsp_context *ctx, const s3dsp_kmap *kmap, int32_t kvol,
                                uint32_t precision, const void *in, uint32_t in_dtype,
                                int64_t n_in, int64_t cin, int32_t in_shift, const void *weight,
                                const float *bias, const void *residual, uint32_t res_dtype,
                                int32_t res_shift, void *out, uint32_t out_dtype, int64_t n_out,
                                int64_t cout, uint32_t flags, const float *pro_sub,
                                const float *pro_mul, const float *pro_add, double *gn_partials,
                                int32_t gn_groups, char *error, uint64_t error_capacity);

/* s3dsp_conv over the channel concat of two tensors, ggml_concat(a, b, 0) of
 * the out_blocks (slat_flow_graph.cpp:466, :497): channels [0, cin_a) of a
 * gathered row come from in_a [n_in, cin_a], channels [cin_a, cin_a + cin_b)
 * from in_b [n_in, cin_b] (the same row of both). The concat is never built:
 * the gather picks the source per channel chunk. weight is packed for
 * cin = cin_a + cin_b; pro_* arrays (F32 strict) index the concat channels.
 * Each width must meet the precision's alignment (BF16: % 8, f32: % 4). */
S3DSP_API s3d_status s3dsp_conv_concat(s3dsp_context *ctx, const s3dsp_kmap *kmap, int32_t kvol,
                                       uint32_t precision, const void *in_a, int64_t cin_a,
                                       const void *in_b, int64_t cin_b, uint32_t in_dtype, int64_t n_in,
                                       int32_t in_shift, const void *weight, const float *bias,
                                       const void *residual, uint32_t res_dtype, int32_t res_shift, void *out,
                                       uint32_t out_dtype, int64_t n_out, int64_t cout, uint32_t flags,
                                       const float *pro_sub, const float *pro_mul, const float *pro_add,
                                       double *gn_partials, int32_t gn_groups, char *error,
                                       uint64_t error_capacity);

/* Name of the kernel s3dsp_conv launches for this shape on ctx's device
 * ("conv_f32_kernel", "conv_tc_kernel" = 128-row tiles, "conv_sk_kernel<256>"
 * / "conv_sk_kernel<128>" = stream-K over 256- / 128-row tiles,
 * "conv_sk_kernel<256>:pairs" = split-K CTA pairs, "conv_halo_kernel" =
 * 128-row tiles with per-tile input halos), or NULL for a NULL ctx / unknown
 * precision. s3dsp_conv_kernel is the in_shift = 0 form (the halo kernel's
 * choice depends on in_shift: a subdivide conv reads few distinct parents).
 * No reference counterpart: a query for profiling and tests. */
S3DSP_API const char *s3dsp_conv_kernel(const s3dsp_context *ctx, int64_t n_out, int32_t kvol, int64_t cin,
                                        int64_t cout, uint32_t precision, uint32_t flags);
S3DSP_API const char *s3dsp_conv_kernel_shift(const s3dsp_context *ctx, int64_t n_out, int32_t kvol, int64_t cin,
                                              int64_t cout, int32_t in_shift, uint32_t precision, uint32_t flags);

/* ---------------------------------------------------------------------------
 * Normalisations (sparse_group_norm mesh_decoder_graph.cpp:16-30;
 * gb_layer_norm graph_builder.cpp:56-62; modulate slat_flow_graph.cpp:55-59).
 * ------------------------------------------------------------------------- */
/* GroupNorm statistics of x [n, c] into f64 partials (same buffer format the
 * conv epilogue writes). */
S3DSP_API s3d_status s3dsp_gn_stats(s3dsp_context *ctx, const void *x, uint32_t dtype, int64_t n,
                                    int64_t c, int32_t groups, double *gn_partials, char *error,
                                    uint64_t error_capacity);
/* Reduces partials into per-channel sub/mul/add such that
 * (x - sub) * mul + add == ((x - mean_g) * rstd_g) * gamma_c + beta_c. */
S3DSP_API s3d_status s3dsp_gn_finalize(s3dsp_context *ctx, const double *gn_partials,
                                       int64_t n_rows, int64_t c, int32_t groups, float eps,
                                       const float *gamma, const float *beta, float *d_sub,
                                       float *d_mul, float *d_add, char *error,
                                       uint64_t error_capacity);
/* y = act((x - sub[c]) * mul[c] + add[c]) with act = SiLU when silu != 0. */
S3DSP_API s3d_status s3dsp_channel_affine(s3dsp_context *ctx, const void *x, uint32_t x_dtype,
                                          int64_t n, int64_t c, const float *sub,
                                          const float *mul, const float *add, int32_t silu,
                                          void *y, uint32_t y_dtype, char *error,
                                          uint64_t error_capacity);
/* Per-row LayerNorm (eps), optional affine gamma/beta, optional modulate
 * h*(1+scale)+shift, optional SiLU. */
S3DSP_API s3d_status s3dsp_layer_norm(s3dsp_context *ctx, const void *x, uint32_t x_dtype,
                                      int64_t n, int64_t c, float eps, const float *gamma,
                                      const float *beta, const float *mod_scale,
                                      const float *mod_shift, int32_t silu, void *y,
                                      uint32_t y_dtype, char *error, uint64_t error_capacity);
/* s3dsp_layer_norm of the channel concat of xa [n, ca] and xb [n, cb] (the
 * out_blocks' norm1 over ggml_concat, slat_flow_graph.cpp:466-477): y
 * [n, ca + cb]; gamma / beta / mod arrays index the concat channels. */
S3DSP_API s3d_status s3dsp_layer_norm_concat(s3dsp_context *ctx, const void *xa, int64_t ca,
                                             const void *xb, int64_t cb, uint32_t x_dtype, int64_t n,
                                             float eps, const float *gamma, const float *beta,
                                             const float *mod_scale, const float *mod_shift, int32_t silu,
                                             void *y, uint32_t y_dtype, char *error,
                                             uint64_t error_capacity);
/* Element type conversion of count elements. */
S3DSP_API s3d_status s3dsp_convert(s3dsp_context *ctx, const void *x, uint32_t x_dtype, void *y,
                                   uint32_t y_dtype, int64_t count, char *error,
                                   uint64_t error_capacity);

/* ---------------------------------------------------------------------------
 * SLat 2x down/up-sample tables and gathers: the coarse half of
 * SlatTables::build (sparse_ops.cpp:53-105, conv_coarse :142) and the
 * downsample / upsample lambdas of slat_flow_graph.cpp:159-190.
 * Coarse rows are the sorted unique (batch, x/2, y/2, z/2) keys (C++
 * truncating division); children are the first 8 fine rows of each coarse
 * cell in fine-row order (sentinel nf); inv_count = 1/(count+1).
 * ------------------------------------------------------------------------- */
S3DSP_API s3d_status s3dsp_slat_tables_build(s3dsp_context *ctx, const s3dsp_hash *fine,
                                             s3dsp_slat_tables **out, char *error,
                                             uint64_t error_capacity);
S3DSP_API void s3dsp_slat_tables_free(s3dsp_context *ctx, s3dsp_slat_tables *tables);
S3DSP_API int64_t s3dsp_slat_tables_coarse_rows(const s3dsp_slat_tables *tables);
/* The coarse submanifold map (conv_coarse); owned by the tables. */
S3DSP_API const s3dsp_kmap *s3dsp_slat_tables_coarse_kmap(const s3dsp_slat_tables *tables);
/* Copies tables to device buffers (any may be NULL): fine_to_coarse [nf],
 * coarse_children [8*nc], coarse_inv_count [nc] f32, coarse_coords [nc, 4]. */
S3DSP_API s3d_status s3dsp_slat_tables_export(s3dsp_context *ctx, const s3dsp_slat_tables *tables,
                                              int32_t *d_fine_to_coarse, int32_t *d_coarse_children,
                                              float *d_coarse_inv_count, int32_t *d_coarse_coords,
                                              char *error, uint64_t error_capacity);
/* y[nc, c] = mean-pool of x[nf, c] (sum of the 8 child slots * inv_count). */
S3DSP_API s3d_status s3dsp_slat_downsample(s3dsp_context *ctx, const s3dsp_slat_tables *tables,
                                           const void *x, uint32_t x_dtype, int64_t c, void *y,
                                           uint32_t y_dtype, char *error, uint64_t error_capacity);
/* y[nf, c] = x[fine_to_coarse[i]] (nearest upsample). */
S3DSP_API s3d_status s3dsp_slat_upsample(s3dsp_context *ctx, const s3dsp_slat_tables *tables,
                                         const void *x, uint32_t x_dtype, int64_t c, void *y,
                                         uint32_t y_dtype, char *error, uint64_t error_capacity);

/* ---------------------------------------------------------------------------
 * Block drivers (host C++ composing the kernels; scratch from the device's
 * stream-ordered pool). Weights are packed for `precision` by
 * s3dsp_weights_pack. Inputs/outputs f32 [rows, channels] on the device.
 * ------------------------------------------------------------------------- */
/* conv3 -> GroupNorm(groups, eps, gamma, beta) -> SiLU -> conv3 -> + x
 * (the config-2 benchmark block; GroupNorm semantics of mesh_decoder_graph.cpp:16-30). */
S3DSP_API s3d_status s3dsp_res_block_gn(s3dsp_context *ctx, const s3dsp_kmap *kmap,
                                        uint32_t precision, const float *x, int64_t n, int64_t c,
                                        const void *w1, const float *b1, const float *gamma,
                                        const float *beta, const void *w2, const float *b2,
                                        int32_t groups, float eps, float *out, char *error,
                                        uint64_t error_capacity);
/* One MeshUpsampleGraph level (mesh_decoder_graph.cpp:42-132): subdivide the
 * parents (hash built with reject_duplicates), GN(32)+SiLU, 27-offset conv
 * over the children reading parent rows, GN(32)+SiLU, 27-offset conv,
 * + 1x1 skip of the parents broadcast to their children. Writes the 8*np
 * child coords and out [8*np, cout]. conv weights MESH_PACKED (27), skip
 * weight 1x1 (LINEAR or SPCONV_1X1), all packed for `precision`. */
S3DSP_API s3d_status s3dsp_mesh_upsample_level(
    s3dsp_context *ctx, const s3dsp_hash *parents, uint32_t precision, const float *x, int64_t cin,
    int64_t cout, const float *gn1_w, const float *gn1_b, const void *conv1_w,
    const float *conv1_b, const float *gn2_w, const float *gn2_b, const void *conv2_w,
    const float *conv2_b, const void *skip_w, const float *skip_b, int32_t *child_coords,
    float *out, char *error, uint64_t error_capacity);
/* The SLat res_block (slat_flow_graph.cpp:216-275): LayerNorm(1e-6, affine)
 * -> SiLU -> conv1 -> LayerNorm(1e-6) -> h*(1+mod_scale)+mod_shift -> SiLU ->
 * conv2 -> + skip (identity, or the Linear skip_w/skip_b when cin != cout).
 * mod_scale/mod_shift [cout] come from the caller's timestep embedding. */
S3DSP_API s3d_status s3dsp_slat_res_block(s3dsp_context *ctx, const s3dsp_kmap *kmap,
                                          uint32_t precision, const float *x, int64_t n,
                                          int64_t cin, int64_t cout, const float *norm1_w,
                                          const float *norm1_b, const void *conv1_w,
                                          const float *conv1_b, const float *mod_scale,
                                          const float *mod_shift, const void *conv2_w,
                                          const float *conv2_b, const void *skip_w,
                                          const float *skip_b, float *out, char *error,
                                          uint64_t error_capacity);
/* The generator's res_block in every form the SLat forward uses
 * (slat_flow_graph.cpp:216-275 for input_blocks.0/1, :463-524 for out_blocks.0/1):
 *   - input: x_a [n_in, cin_a], or the channel concat of x_a and x_b
 *     [n_in, cin_b] (x_b NULL, cin_b 0 for one source), f32;
 *   - up_rows NULL: n_in == kmap rows (input_blocks, out_blocks.1);
 *     up_rows int32 [kmap rows]: the block runs at the fine resolution of
 *     `kmap` on the nearest upsample of its coarse input (out_blocks.0,
 *     upsample at :467 = get_rows by fine_to_coarse, :185-190); the
 *     upsampled tensor is never built -- norm1 and the skip Linear run on
 *     the coarse rows (both are row-wise) and conv1 gathers coarse rows
 *     through the kernel map composed with up_rows;
 *   - skip: identity when one source, no upsample and cin == cout; otherwise
 *     the Linear skip_w/skip_b (packed LINEAR for cin_a + cin_b -> cout).
 * out [kmap rows, cout] f32. Entries of up_rows outside [0, n_in) are read
 * as "no row" and reported by the next status check. */
S3DSP_API s3d_status s3dsp_slat_res_block_concat(
    s3dsp_context *ctx, const s3dsp_kmap *kmap, const int32_t *up_rows, uint32_t precision, const float *x_a,
    int64_t cin_a, const float *x_b, int64_t cin_b, int64_t n_in, int64_t cout, const float *norm1_w,
    const float *norm1_b, const void *conv1_w, const float *conv1_b, const float *mod_scale,
    const float *mod_shift, const void *conv2_w, const float *conv2_b, const void *skip_w, const float *skip_b,
    float *out, char *error, uint64_t error_capacity);
/* Host-buffer forms (what decode_object_mesh does per level with its Backend,
 * session.cpp:927-962): upload coords + features, build the tables, run the
 * block, read the result back. Synchronous. */
S3DSP_API s3d_status s3dsp_res_block_gn_host(s3dsp_context *ctx, uint32_t precision,
                                             const int32_t *h_coords, int64_t n, const float *h_x,
                                             int64_t c, const void *w1, const float *b1,
                                             const float *gamma, const float *beta, const void *w2,
                                             const float *b2, int32_t groups, float eps,
                                             float *h_out, char *error, uint64_t error_capacity);
/* s3dsp_res_block_gn_host without the wait: the copies in, the tables, the
 * block and the copy out are queued on the context's stream and the call
 * returns; h_out holds the result once that stream reaches the end of this
 * work (synchronise the stream or an event recorded after the call). Needs a
 * context created with S3DSP_CONTEXT_DEFERRED_CHECKS (device-detected input
 * errors are read by s3dsp_context_check). The host buffers must stay valid
 * until then; pinned host memory lets the copies of one call overlap another
 * context's kernels, which is how one host thread keeps several contexts
 * busy. On a context with S3DSP_CONTEXT_COPY_STREAMS the copies run on the
 * context's copy streams instead, and h_out holds the result once the
 * copy-out stream gets there (s3dsp_context_join, then the stream; or
 * s3dsp_context_check). No counterpart in the reference (its Backend::run is
 * synchronous, backend.hpp:16-92). */
S3DSP_API s3d_status s3dsp_res_block_gn_host_queued(s3dsp_context *ctx, uint32_t precision,
                                                    const int32_t *h_coords, int64_t n, const float *h_x,
                                                    int64_t c, const void *w1, const float *b1,
                                                    const float *gamma, const float *beta, const void *w2,
                                                    const float *b2, int32_t groups, float eps, float *h_out,
                                                    char *error, uint64_t error_capacity);
S3DSP_API s3d_status s3dsp_mesh_upsample_level_host(
    s3dsp_context *ctx, uint32_t precision, const int32_t *h_parent_coords, int64_t np,
    const float *h_x, int64_t cin, int64_t cout, const float *gn1_w, const float *gn1_b,
    const void *conv1_w, const float *conv1_b, const float *gn2_w, const float *gn2_b,
    const void *conv2_w, const float *conv2_b, const void *skip_w, const float *skip_b,
    int32_t *h_child_coords, float *h_out, char *error, uint64_t error_capacity);

#ifdef __cplusplus
}
#endif

#endif /* S3DSP_H */
