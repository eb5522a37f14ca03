/*
 * p3d.h — C ABI of the B200-native (sm_100a) sparse-voxel SLat kernel library
 * (libp3dcuda.so).
 *
 * This is the drop-in boundary for the hot path of Pixal3D.cpp: the
 * SparseTensor ops of src/sparse.cpp, the sparse transformer block of
 * src/sparse_transformer.cpp, their use by src/slat_flow.cpp and
 * src/slat_decoder.cpp, and the Euler/CFG loop of src/flow_sampler.cpp.
 * Each entry point below names the reference interface it replaces
 * (path:line inside the Pixal3D.cpp project).  The C++17 host layer
 * (pixal3d/cpp_b200/host/) implements the reference's own
 * include/pixal3d/{sparse,sparse_transformer,flow_sampler,slat_flow,
 * slat_decoder}.h signatures on top of these calls.
 *
 * Conventions
 *  - All tensor arguments are DEVICE pointers on the context's device; the
 *    caller owns them.  Calls are stream-ordered on the context's stream and
 *    return a p3d_status (0 = OK).  p3d_last_error() gives the message.
 *  - coords: int32 [n][4] rows (batch, x, y, z), rows contiguous by batch.
 *  - feats: row-major [n][channels]; 16-bit operands are raw uint16 bit
 *    patterns of IEEE bfloat16 or binary16 as the call's dtype argument says.
 *  - Linear weights [out][in]; conv weights [27][out][in] with
 *    kernel = kd*9 + kh*3 + kw and offset (kd-1, kh-1, kw-1) on (x, y, z).
 *  - Neighbour maps: int32 [27][n], missing neighbour = n.
 *  - Device-side faults that a kernel can detect (hash probe bound,
 *    duplicate coordinate, bounded-wait timeout) are latched in a per-context
 *    device flag; p3d_ctx_check() synchronizes and reports it.
 */
#ifndef P3D_H
#define P3D_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum p3d_status {
    P3D_OK = 0,
    P3D_ERR_INVALID = 1,      /* bad argument: null pointer, shape, alignment */
    P3D_ERR_CUDA = 2,         /* CUDA runtime error */
    P3D_ERR_HASH_FULL = 3,    /* coordinate hash probe bound exceeded */
    P3D_ERR_TIMEOUT = 4,      /* a device-side bounded wait expired */
    P3D_ERR_UNSUPPORTED = 5,  /* shape outside what the kernels implement */
    P3D_ERR_NO_DEVICE = 6,    /* no sm_100 device */
    P3D_ERR_DUPLICATE = 7,    /* duplicate coordinate in a sparse tensor */
    P3D_ERR_NONFINITE = 8     /* non-finite value found by a validity probe */
};

/* Element types.  GEMM/conv/attention operands are 16-bit (bf16 or f16, both
 * on the tensor cores with f32 accumulation); f32 is used for residual
 * streams, statistics and model outputs. */
enum p3d_dtype { P3D_F32 = 0, P3D_BF16 = 1, P3D_F16 = 2 };

/* GEMM / conv epilogues (bit flags; at most one activation). */
enum p3d_epilogue {
    P3D_EPI_NONE = 0,
    P3D_EPI_GELU_TANH = 1,   /* out = gelu_tanh(acc + bias) */
    P3D_EPI_SILU = 2,        /* out = silu(acc + bias) */
    P3D_EPI_RESIDUAL = 4     /* out(f32) += gate[batch(row)] * (acc + bias) */
};

typedef struct p3d_ctx p3d_ctx;

/* ---------------------------------------------------------------- context */

/* Create a context on `device` using `stream` (cudaStream_t, may be NULL for
 * the legacy default stream).  No reference counterpart: replaces the
 * ggml backend/scheduler plumbing of src/backend.cpp for this path.
 * The caller's current device is left unchanged.  Kernel entry points
 * expect ctx's device to be current (as CUDA runtime calls do); the
 * p3d_flow_* entry points make it current themselves for their duration. */
int p3d_ctx_create(int device, void *stream, p3d_ctx **out);
int p3d_ctx_destroy(p3d_ctx *ctx);
int p3d_ctx_set_stream(p3d_ctx *ctx, void *stream);
void *p3d_ctx_stream(const p3d_ctx *ctx);
/* Message of the last failed call on this context ("" if none). */
const char *p3d_last_error(const p3d_ctx *ctx);
/* Synchronize the stream and report (then clear) the device fault flag. */
int p3d_ctx_check(p3d_ctx *ctx);
/* Number of kernels this library launched on ctx since creation. */
int64_t p3d_ctx_launch_count(const p3d_ctx *ctx);
int p3d_version(void);

/* Device buffers and copies on ctx's device and stream (the "device sparse
 * tensor create/upload/download" of the boundary; no reference counterpart:
 * the reference's tensors are host std::vectors).  p3d_copy_to_device is
 * stream-ordered; p3d_copy_to_host returns after the data has arrived. */
int p3d_device_alloc(p3d_ctx *ctx, size_t bytes, void **out);
int p3d_device_free(p3d_ctx *ctx, void *ptr);
int p3d_copy_to_device(p3d_ctx *ctx, void *dst, const void *src, size_t bytes);
int p3d_copy_to_host(p3d_ctx *ctx, void *dst, const void *src, size_t bytes);
/* Wait for ctx's stream, then report (and clear) a latched device fault. */
int p3d_ctx_synchronize(p3d_ctx *ctx);

/* No reference counterpart: a check of the failure path that every
 * pipeline wait of this library takes.  One device thread waits, through the
 * same bounded-wait routine the kernels use, on an mbarrier phase; with
 * complete != 0 another warp completes it, with complete == 0 nothing does
 * and the wait gives up after limit_ns (at most 5 s).  Synchronizes, writes
 * out_host[0] = 1 if the wait succeeded (else 0) and out_host[1] = the
 * wait's duration in ns, and returns p3d_ctx_check's status: P3D_ERR_TIMEOUT
 * after an expired wait (the flag is then cleared and ctx stays usable). */
int p3d_wait_selftest(p3d_ctx *ctx, int complete, int64_t limit_ns, int64_t *out_host);

/* ------------------------------------------------------ coordinates/hash */

/* Table slots for n keys (power of two >= 2n).  Keys are uint64, values
 * int32; the caller allocates both arrays of this length. */
int64_t p3d_coord_hash_capacity(int64_t n);

/* Insert every row of coords into an open-addressing table in HBM
 * (warp-cooperative bucketed linear probing: 4 lanes of a warp per key read
 * a window of 4 slots, one 32-byte sector, per step; bounded probes).  Keys pack 16 bits per
 * field, so batch must lie in [0, 65536) and x, y, z in [-32768, 32768): a
 * row outside that range latches P3D_ERR_INVALID instead of aliasing
 * another key, and p3d_neighbor_map27 reports neighbours outside it as
 * missing.  capacity: a power of two >= max(n, 64).  Replaces the
 * std::unordered_map<Coord,size_t,CoordHash> builds in
 * src/sparse.cpp:1017-1022 and src/slat_decoder.cpp:630-635.  A duplicate
 * coordinate latches P3D_ERR_DUPLICATE (SparseTensorF32::valid,
 * src/sparse.cpp:318-321). */
int p3d_coord_hash_build(p3d_ctx *ctx, const int32_t *coords, int64_t n, uint64_t *table_keys,
                         int32_t *table_vals, int64_t capacity);

/* 27-offset gather map [27][n], sentinel n.  Replaces
 * build_neighbor_gather_map / build_reference_neighbor_gather_map
 * (src/slat_decoder.cpp:609-714); bit-exact with the reference. */
int p3d_neighbor_map27(p3d_ctx *ctx, const int32_t *coords, int64_t n, const uint64_t *table_keys,
                       const int32_t *table_vals, int64_t capacity, int32_t *nbr_out);

/* Bytes of scratch p3d_neighbor_map27_ws needs for n points. */
size_t p3d_neighbor_map27_workspace(int64_t n);
/* Hash build + neighbour map in one call, using caller scratch `ws` of
 * p3d_neighbor_map27_workspace(n) bytes (256-byte aligned). */
int p3d_neighbor_map27_ws(p3d_ctx *ctx, const int32_t *coords, int64_t n, void *ws, size_t ws_bytes,
                          int32_t *nbr_out);

/* Device validity probe of a sparse tensor (SparseTensorF32::valid,
 * src/sparse.cpp:261-335; VarLenTensorF32::valid's finiteness scan,
 * :213-239 when coords is NULL).  Writes to *first_bad (device int64) the
 * first failing row and check as (row << 2 | code), code 0 = coordinate
 * outside [0,batch) x [0,sx) x [0,sy) x [0,sz), 1 = duplicate of an earlier
 * row, 2 = batch index decreasing, 3 = non-finite feature; or a value
 * >= 0x7F7F7F7F7F7F7F7F when the tensor is valid.  This is the error the
 * reference's sequential scan reports.  feats may be NULL (coordinates
 * only).  ws: p3d_sparse_validate_workspace(n) bytes, 256-byte aligned
 * (unused when coords is NULL).  With coords, batch above 65536 or an extent
 * above 32768 is P3D_ERR_UNSUPPORTED (the hash key's field range). */
size_t p3d_sparse_validate_workspace(int64_t n);
int p3d_sparse_validate(p3d_ctx *ctx, const int32_t *coords, int64_t n, const float *feats, int channels,
                        int batch, int sx, int sy, int sz, void *ws, size_t ws_bytes, int64_t *first_bad);

/* No counterpart in the reference.  The output of p3d_neighbor_map27_ws,
 * for callers that cannot allocate device memory: a device node inside a
 * planned graph (a ggml custom op, whose graph allocator sizes every tensor
 * before compute and hands the node only its inputs and outputs), or a host
 * that binds only this C ABI and owns no device allocator.  The hash table
 * is a 12 MiB file-scope device array (2^20 slots) that every GPU which
 * loads the library holds until the process exits; the call makes no
 * cudaMalloc/cudaFree and no allocating library call.
 *   - n above P3D_NBR_STATIC_MAX_POINTS is rejected with P3D_ERR_INVALID.
 *   - Every call looks up the array's address on ctx's device
 *     (cudaGetSymbolAddress, with that device current), so the address is
 *     never stale, even after a device reset.  The first call on a device
 *     also loads the library's device code there: make that first call
 *     before any stream capture.
 *   - Every call shares the one array and clears the slots it uses; calls
 *     that overlap on the GPU (other streams, contexts or threads on the
 *     same device) race on it and must be serialised by the caller. */
#define P3D_NBR_STATIC_MAX_POINTS 524288
int p3d_neighbor_map27_static(p3d_ctx *ctx, const int32_t *coords, int64_t n, int32_t *nbr_out);

/* Downsample topology (sparse_downsample_mean, src/sparse.cpp:536-602):
 * parents = coords / factor (per batch), output rows sorted
 * lexicographically by (b,x,y,z) like the reference.  Uses a dense
 * occupancy grid of batch*ceil(sx/f)*ceil(sy/f)*ceil(sz/f) int32 cells in
 * `grid` (caller scratch).  Writes out_coords [m][4], parent[n] (output row
 * of each input row), child[m][f^3] (input row of each child octant or -1,
 * octant = (x%f)*f*f + (y%f)*f + z%f) and *out_m (device int64).  `grid` holds
 * p3d_downsample_grid_ints(...) int32.
 * out_coords/child must hold n rows (m <= n). */
int p3d_downsample_topology(p3d_ctx *ctx, const int32_t *coords, int64_t n, int batch, int sx, int sy,
                            int sz, int factor, int32_t *grid, int32_t *out_coords, int32_t *parent,
                            int32_t *child, int64_t *out_m);
/* int32 cells of `grid` scratch p3d_downsample_topology needs. */
int64_t p3d_downsample_grid_ints(int batch, int sx, int sy, int sz, int factor);
/* Mean of children features (f32 or bf16 in, same dtype out), summed in
 * octant order == the reference's input-row order for sorted input. */
int p3d_downsample_mean(p3d_ctx *ctx, const void *x, int64_t m, int channels, int factor,
                        const int32_t *child, int dtype, void *out);
/* Nearest 2x upsample (no reference; benchmark config 2): out[i] = x[parent[i]]. */
int p3d_upsample_nearest(p3d_ctx *ctx, const void *x, int64_t n, int channels, const int32_t *parent,
                         int dtype, void *out);

/* Channel-to-spatial topology (sparse_channel_to_spatial,
 * src/sparse.cpp:604-702): child c of parent p is kept when mask is NULL or
 * mask[p*f^3 + c] > 0; output rows in parent order then child order.
 * Writes out_coords (n*f^3 rows max), src_row/src_child per output row and
 * *out_m (device int64).  scratch: n+1 int64. */
int p3d_c2s_topology(p3d_ctx *ctx, const int32_t *coords, int64_t n, int factor, const float *mask,
                     int64_t *scratch, int32_t *out_coords, int32_t *src_row, int8_t *src_child,
                     int64_t *out_m);
/* Feature half of channel-to-spatial: out[j] = x[src_row[j], src_child[j]*cout : +cout],
 * optionally repeating each channel `repeat` times (repeat_channels,
 * src/slat_decoder.cpp:80-109). */
/* offsets[b] = first row of batch item b in a batch-contiguous coordinate
 * list, offsets[batch] = n (the per-item row ranges every batch-aware call
 * takes).  offsets: device int32 [batch + 1]. */
int p3d_batch_offsets(p3d_ctx *ctx, const int32_t *coords, int64_t n, int batch, int32_t *offsets);
int p3d_c2s_gather(p3d_ctx *ctx, const void *x, int64_t in_channels, const int32_t *src_row,
                   const int8_t *src_child, int64_t m, int cout, int repeat, int dtype, void *out);

/* ------------------------------------------------------------ contractions */

/* y = epilogue(x W^T + bias) on tcgen05/TMEM tensor cores, TMA-fed, 16-bit
 * operands (ab_dtype P3D_BF16 or P3D_F16), f32 accumulation.  Replaces
 * sparse_linear / varlen_linear / row_linear (src/sparse.cpp:337-488,
 * src/slat_flow.cpp:85-111).
 * x: [m][ldx] (k used), w: [n][k], bias f32 [n] or NULL.
 * out: [m][ldo] of out_dtype.  For P3D_EPI_RESIDUAL out must be f32 and is
 * updated in place: out += g * (acc + bias), g = gate[b*gate_ld + col] with
 * b the batch of the row from batch_offsets[nbatch+1] (or 1 if gate NULL).
 * Requires k % 8 == 0, ldx % 8 == 0, 16-byte aligned x/w. */
int p3d_linear(p3d_ctx *ctx, const void *x, int64_t ldx, const void *w, int ab_dtype, const float *bias, int64_t m,
               int64_t n, int64_t k, void *out, int64_t ldo, int out_dtype, int epilogue,
               const float *gate, int64_t gate_ld, const int32_t *batch_offsets, int nbatch);

/* p3d_linear with the per-head query/key normalisation of the attention
 * blocks fused into its epilogue (head_dim 64): after the bias, columns
 * [0, norm_cols) are RMS-normalised per 64-column head with gamma[col]
 * (sparse_multihead_rms_norm, src/sparse.cpp:919-954), and columns
 * [0, rope_cols) are rotated by the interleaved 3D RoPE with
 * rope_table[pair][row] = (cos, sin), 32 pairs x m rows, from p3d_rope_table
 * (sparse_rotary_position_embedding, src/sparse.cpp:861-917).  Normalises
 * the f32 accumulators before rounding to out_dtype.  n, norm_cols and
 * rope_cols must be multiples of 64. */
int p3d_linear_headnorm(p3d_ctx *ctx, const void *x, int64_t ldx, const void *w, int ab_dtype,
                        const float *bias, int64_t m, int64_t n, int64_t k, void *out, int64_t ldo,
                        int out_dtype, int64_t norm_cols, const float *gamma, int64_t rope_cols,
                        const float *rope_table);

/* Submanifold 3x3x3 sparse conv as one gather-GEMM on tcgen05 tiles:
 * out[p] = epilogue(bias + sum_k W[k] x[nbr[k][p]]).  Replaces
 * sparse_submanifold_conv3d (src/sparse.cpp:999-1055) and the ggml
 * get_rows/mul_mat chain gpu_sparse_conv_node (src/slat_decoder.cpp:855-906).
 * x [n][cin] (cin % 64 == 0), w [27][cout][cin], both of ab_dtype.
 * Epilogues as p3d_linear (RESIDUAL adds into f32 out). */
int p3d_subm_conv3d(p3d_ctx *ctx, const void *x, int64_t n, int64_t cin, const int32_t *nbr,
                    const void *w, int ab_dtype, const float *bias, int64_t cout, void *out, int64_t ldo,
                    int out_dtype, int epilogue, const float *gate, int64_t gate_ld,
                    const int32_t *batch_offsets, int nbatch);

/* The same conv with the taps of each 256-row tile given: bit t of
 * tile_taps[b] set when some row of rows [256 b, 256 b + 256) has a
 * neighbour at tap t (p3d_conv_tile_taps).  The CTA-pair kernel (cout a
 * multiple of 256) skips the other taps, whose gathered rows are all zero,
 * so the result equals p3d_subm_conv3d's bit for bit; other shapes ignore
 * tile_taps.  Rows ordered so that tiles share their missing taps (for a
 * surface, by neighbour pattern) skip the most.  tile_taps NULL = every tap. */
int p3d_subm_conv3d_taps(p3d_ctx *ctx, const void *x, int64_t n, int64_t cin, const int32_t *nbr, const void *w,
                         int ab_dtype, const float *bias, int64_t cout, void *out, int64_t ldo, int out_dtype,
                         int epilogue, const float *gate, int64_t gate_ld, const int32_t *batch_offsets, int nbatch,
                         const uint32_t *tile_taps);
/* tile_taps [ceil(n / 256)] of a neighbour map [27][n] (missing = n). */
int p3d_conv_tile_taps(p3d_ctx *ctx, const int32_t *nbr, int64_t n, uint32_t *tile_taps);

/* Row order under which conv tiles share their missing taps (no reference
 * counterpart: a layout choice of this library's conv): perm[i] = the row
 * at position i when the rows are stably sorted by (batch index, chunk,
 * neighbour pattern).  chunk = row / chunk_rows in the input order (one
 * chunk when chunk_rows <= 0), so a spatially ordered input (e.g. raster
 * order) keeps its locality at chunk scale while rows of one chunk are
 * grouped by pattern; the pattern's bit t is set when nbr[t][row] < n.  A
 * stable device radix sort, so equal keys keep their input order.  coords
 * [n][4] (batch in [0, batch)), nbr [27][n] of those coords; ws:
 * p3d_conv_row_order_workspace(n, batch, chunk_rows) bytes (0 when the key
 * would not fit 64 bits), 256-byte aligned.  Run a conv in this order by
 * gathering the coordinates (and input rows) through perm and building the
 * neighbour map of the reordered coordinates. */
#define P3D_CONV_ORDER_CHUNK_ROWS 4096 /* chunk_rows of the flow's fine-level conv order */
size_t p3d_conv_row_order_workspace(int64_t n, int batch, int64_t chunk_rows);
int p3d_conv_row_order(p3d_ctx *ctx, const int32_t *coords, const int32_t *nbr, int64_t n, int batch,
                       int64_t chunk_rows, void *ws, size_t ws_bytes, int32_t *perm);

/* Varlen flash attention on tcgen05 tensor cores, head_dim 64, 16-bit in/out
 * (dtype), f32 softmax/accumulation.  rows_q / rows_k: total rows of the q and
 * k/v views (cu_q[nseq], cu_k[nseq]); q/k/v/out rows 16-byte aligned.
 * Sequence s covers q rows [cu_q[s], cu_q[s+1]) and k/v rows
 * [cu_k[s], cu_k[s+1]).  Replaces sparse_scaled_dot_product_attention
 * (src/sparse.cpp:704-783), sparse_cross_attention (:785-859) and the
 * chunked ggml sdpa of src/slat_flow.cpp:947-1001. */
int p3d_varlen_attention(p3d_ctx *ctx, const void *q, int64_t ldq, const void *k, int64_t ldk,
                         const void *v, int64_t ldv, void *out, int64_t ldo, const int32_t *cu_q,
                         const int32_t *cu_k, int nseq, int64_t max_q, int64_t rows_q, int64_t rows_k,
                         int heads, int head_dim, float scale, int dtype);

/* Shifted-window sparse self-attention (no reference implementation: the
 * 8^3-window blocks of the config-3 SLat decoder).  Row i with coords
 * (b, x, y, z) lies in window (b, (x+shift)/window, (y+shift)/window,
 * (z+shift)/window) of a grid with ceil((s_d + shift)/window) windows per
 * axis; window index w = ((b*nwx + wx)*nwy + wy)*nwz + wz.
 * p3d_window_count: batch*nwx*nwy*nwz (0 for bad arguments).
 * p3d_window_partition: perm[j] = row at window-order position j (rows
 * ordered by window, then by row index; -1 marks a position left empty by a
 * row outside [0, batch) x grid, which also latches P3D_ERR_INVALID), and
 * cu[w] = first position of window w, cu[num_windows] = number of rows
 * placed.  window^3 <= 1024, 0 <= shift < window.  ws: at least
 * p3d_window_partition_workspace(n, num_windows) bytes. */
int64_t p3d_window_count(int batch, int window, int shift, int sx, int sy, int sz);
size_t p3d_window_partition_workspace(int64_t n, int64_t num_windows);
int p3d_window_partition(p3d_ctx *ctx, const int32_t *coords, int64_t n, int batch, int window, int shift, int sx,
                         int sy, int sz, int32_t *perm, int32_t *cu, void *ws, size_t ws_bytes);
/* Attention of every row to the rows of its window (the partition above):
 * q/k/v rows gathered into window order, p3d_varlen_attention semantics per
 * window (head_dim 64, 16-bit dtype), output rows written back in the
 * canonical order (out row i belongs to input row i).  max_window_rows
 * bounds the rows of one window (window^3).  scratch: at least
 * p3d_window_attention_scratch(n, heads) bytes, 16-byte aligned. */
size_t p3d_window_attention_scratch(int64_t n, int heads);
int p3d_window_attention(p3d_ctx *ctx, const void *q, int64_t ldq, const void *k, int64_t ldk, const void *v,
                         int64_t ldv, const int32_t *perm, const int32_t *cu, int64_t num_windows,
                         int max_window_rows, int64_t n, int heads, int head_dim, float scale, int dtype,
                         void *scratch, size_t scratch_bytes, void *out, int64_t ldo);

/* ---------------------------------------------------- SLat cascade glue */

/* Latent (de)normalization of a SLat stage (normalize_slat_f32,
 * src/pipeline.cpp:333-357; the denormalization of run_slat_stage_f32,
 * :418-431): out[i][c] = (x[i][c] - mean[c]) / std[c], or with denormalize
 * x[i][c] * std[c] + mean[c], f32 with the reference's rounding (bit-exact).
 * x, out f32 [n][channels] (may alias); mean, std f32 [channels] on the
 * device.  A non-finite result latches P3D_ERR_NONFINITE. */
int p3d_slat_normalize(p3d_ctx *ctx, const float *x, int64_t n, int channels, const float *mean, const float *std,
                       int denormalize, float *out);

/* Shape-decoder coordinates to the 1024 cascade grid
 * (quantize_slat_coords_f32, src/pipeline.cpp:433-466): each axis v of
 * coords [n][4] (batch b in [0, batch)) maps to llround((v + 0.5) /
 * low_resolution * 63) in double; rows are made unique and written in
 * lexicographic (b, x, y, z) order to out (capacity n rows); *count (device
 * int64) receives the number of rows.  resolution must be 1024 ("SLat
 * cascade resolution must be 1024"); a coordinate mapping outside [0, 64)
 * latches P3D_ERR_INVALID.  ws: p3d_quantize_slat_coords_workspace(batch)
 * bytes; all pointers 16-byte aligned.  The max_num_tokens guard of the
 * reference is the caller's check of *count. */
size_t p3d_quantize_slat_coords_workspace(int batch);
int p3d_quantize_slat_coords(p3d_ctx *ctx, const int32_t *coords, int64_t n, int batch, int low_resolution,
                             int resolution, int32_t *out, int64_t *count, void *ws, size_t ws_bytes);

/* ------------------------------------------------- projection conditioning */

/* One camera view of an image feature map (ProjectionView plus the view's
 * ProjectionGridOptions::image_resolution, include/pixal3d/projection.h:13-55).
 * feature_map: DEVICE f32 [height][width][channels], row-major.  The camera
 * is the canonical front view at `distance` unless has_transform, in which
 * case transform_matrix is the row-major camera-to-world matrix. */
typedef struct p3d_projection_view {
    const float *feature_map;
    int height, width, channels;
    int image_resolution;
    float camera_angle_x, distance, mesh_scale;
    int has_transform;
    float transform_matrix[16];
} p3d_projection_view;

/* Project points of a grid_resolution^3 grid into each view and sample its
 * map with grid_sample's bilinear / align_corners=False / border rules.
 * coords: sparse rows (0, x, y, z) with 0 <= x, y, z < grid_resolution
 * (project_grid_features_at_coords, src/projection.cpp:359-434), or NULL
 * for all n == grid_resolution^3 cells in meshgrid "ij" order
 * (project_grid_features, :342-357).  With nviews > 1 (at most 8, equal
 * channel counts) the output is the f32 sum over views in order times
 * 1/nviews (project_grid_features_average, :436-481; the per-view sum of
 * project_condition_stage_multiview_average_f32, src/condition.cpp:
 * 878-940).  out: [n][ldo] f32/bf16/f16, columns [0, channels) written, so a
 * second call at out + channels appends another map's channels (the DINO |
 * NAF concatenation of src/condition.cpp:797-812).  valid: u8 [n] or NULL,
 * 1 where some view projects the point inside the image and in front of the
 * camera.  Features and flags equal the reference's f32 CPU results bit for
 * bit.  Option / camera errors carry the reference's messages; a coordinate
 * outside the grid latches P3D_ERR_INVALID (its row is written as zeros).
 * n == 0 validates the views and options only. */
int p3d_project_features(p3d_ctx *ctx, const p3d_projection_view *views, int nviews, int grid_resolution,
                         const int32_t *coords, int64_t n, void *out, int64_t ldo, int out_dtype,
                         uint8_t *valid);

/* Host math, no device work: relative[i] = F(distances[0]) *
 * inverse(c2w[0]) * c2w[i] for row-major 4x4 matrices (HOST pointers,
 * c2w/relative [nviews][16]); compute_relative_calc_matrices,
 * src/projection.cpp:528-561.  ctx may be NULL (no message kept). */
int p3d_projection_relative_matrices(p3d_ctx *ctx, const float *c2w, const float *distances, int nviews,
                                     float *relative);

/* ------------------------------------------------------ fused elementwise */

/* x[i, c] += sinusoidal absolute 3D position embedding of coords[i] (no
 * reference: the configs' "sinusoidal 3D absolute PE"): with fd = channels/6
 * frequencies f_j = 10000^(-j/fd), axis a (x, y, z) fills channels
 * [2*fd*a, 2*fd*a + fd) with sin(coord_a * f_j) and the next fd with cos;
 * channels >= 6*fd are left unchanged.  x: f32 [n, channels]. */
int p3d_ape_add(p3d_ctx *ctx, const int32_t *coords, int64_t n, int channels, float *x);

/* LayerNorm over channels of f32 rows (two-pass, like sparse_layer_norm,
 * src/sparse.cpp:490-534), then optional affine (gamma/beta) and optional
 * AdaLN modulation y*(1+scale[b])+shift[b] with shift = mod[b*mod_ld + c],
 * scale = mod[b*mod_ld + C + c] (affine_modulate,
 * src/sparse_transformer.cpp:71-99).  out bf16 or f32. */
int p3d_layernorm_modulate(p3d_ctx *ctx, const float *x, int64_t n, int channels, float eps,
                           const float *gamma, const float *beta, const float *mod, int64_t mod_ld,
                           const int32_t *batch_offsets, int nbatch, void *out, int out_dtype);

/* Per-head RMS norm (sparse_multihead_rms_norm, src/sparse.cpp:919-997) and
 * optional interleaved 3D RoPE (sparse_rotary_position_embedding,
 * src/sparse.cpp:861-917) in place on 16-bit rows x[n][ld] (heads*head_dim
 * used).  gamma may be NULL (no norm); coords NULL means no RoPE. */
int p3d_qk_rmsnorm_rope(p3d_ctx *ctx, void *x, int64_t n, int64_t ld, int heads, int head_dim,
                        const float *gamma, const int32_t *coords, float freq_min, float freq_base,
                        int dtype);
/* Per-point RoPE cos/sin table for p3d_linear_headnorm
 * (src/sparse.cpp:881-906), pair-major: table[p][i] = (cos, sin) of pair p
 * of point i (float2 [head_dim/2][n]); pairs past 3*floor(head_dim/6) get
 * (1, 0). */
int p3d_rope_table(p3d_ctx *ctx, const int32_t *coords, int64_t n, int head_dim, float freq_min,
                   float freq_base, float *table);

/* LayerNorm (+affine when gamma/beta) (+SiLU when silu != 0) written to an
 * operand of row pitch ld_out >= channels, padding columns zeroed
 * (sparse_layer_norm + silu_in_place, src/sparse.cpp:490-534,
 * src/slat_decoder.cpp:68-78).  x f32 [n][channels]. */
int p3d_layernorm_act(p3d_ctx *ctx, const float *x, int64_t n, int channels, float eps, const float *gamma,
                      const float *beta, int silu, void *out, int64_t ld_out, int out_dtype);
/* f32 [rows][cols] -> out_dtype [rows][ld] (ld >= cols, padding zeroed): the
 * 16-bit GEMM operand layout.  No reference counterpart (layout plumbing). */
int p3d_pack_operand(p3d_ctx *ctx, const float *x, int64_t rows, int cols, void *out, int64_t ld, int out_dtype);

/* Head-width repack (no reference counterpart; layout plumbing for head_dim
 * below the attention kernel's 64): out[r][h][c] = x[r][h][c] for
 * c < min(hd_in, hd_out), 0 for the rest of the hd_out columns, and the
 * row padding out[r][heads*hd_out .. ldo) = 0 (whole rows of out written).
 * x and out must not overlap. */
int p3d_repack_heads(p3d_ctx *ctx, const void *x, int64_t ldx, int64_t n, int heads, int hd_in, int hd_out,
                     void *out, int64_t ldo, int dtype);

/* out = act(x) elementwise (gelu_tanh_in_place src/sparse_transformer.cpp:123-134;
 * silu src/slat_decoder.cpp:68-78).  dtype applies to x and out. */
int p3d_activation(p3d_ctx *ctx, const void *x, int64_t count, int act, int dtype, void *out);

/* GroupNorm over the points of each batch item (no reference; benchmark
 * config 2 SparseResBlock3d), then optional SiLU; f32 in, f32/bf16/f16 out.
 * channels/groups must be a multiple of 4; x/out 16-byte aligned.
 * stats: caller scratch of nbatch*groups*3 doubles. */
int p3d_group_norm_silu(p3d_ctx *ctx, const float *x, int64_t n, int channels, int groups, float eps,
                        const float *gamma, const float *beta, const int32_t *batch_offsets, int nbatch,
                        int silu, double *stats, void *out, int out_dtype);

/* Euler/CFG update of flow_euler_sample_f32 (src/flow_sampler.cpp:245-343):
 * pred = g*v_pos + (1-g)*v_neg (or v_pos when v_neg NULL), optional guidance
 * rescale (src/flow_sampler.cpp:200-241) with per-batch population std,
 * then x -= (t - t_next) * pred.  x, v_*: f32 [n][c]; stats scratch of
 * nbatch*4 doubles.  x0_out (optional, [n][c]): the step's predicted x0,
 * pred_to_xstart(x, t, pred) (src/flow_sampler.cpp:139-147), for trajectories. */
int p3d_euler_cfg_step(p3d_ctx *ctx, float *x, const float *v_pos, const float *v_neg, int64_t n,
                       int channels, const int32_t *batch_offsets, int nbatch, float t, float t_next,
                       float guidance, float guidance_rescale, float sigma_min, double *stats,
                       float *x0_out);

/* Precision conversion between any two p3d_dtype element types. */
int p3d_convert(p3d_ctx *ctx, const void *x, int x_dtype, int64_t count, void *out, int out_dtype);

/* ------------------------------------------------------- SLat flow model */

/* Hyper-parameters (SLatFlowHParams, include/pixal3d/slat_flow.h:12-37) plus
 * the benchmark-config extensions with no reference: pe_mode 1 = sinusoidal
 * absolute 3D PE, io_resblocks > 0 = SparseResBlock3d input/output stages
 * around a 2x downsample/upsample of the trunk. */
typedef struct p3d_flow_hparams {
    int in_channels, out_channels, model_channels, cond_channels;
    int num_blocks, num_heads, mlp_hidden, proj_in_channels;
    int proj_mode;     /* image_attn_mode: 0 cross, 1 proj */
    int qk_rms_norm, qk_rms_norm_cross;
    int pe_mode;       /* 0 rope, 1 ape */
    int io_resblocks;  /* 0 = reference model */
    int groups;        /* GroupNorm groups for io resblocks */
    int operand_dtype; /* 16-bit GEMM/attention operand type: P3D_F16 or P3D_BF16 */
    float norm_eps, rope_freq_min, rope_freq_base;
} p3d_flow_hparams;

/* Per-block weight pointers, f32, DEVICE memory, in
 * SparseTransformerBlockWeightsF32 order (include/pixal3d/sparse_transformer.h:30-54). */
typedef struct p3d_block_weights {
    const float *modulation, *qkv_w, *qkv_b, *q_gamma, *k_gamma, *out_w, *out_b;
    const float *norm2_w, *norm2_b, *cq_w, *cq_b, *ckv_w, *ckv_b, *cq_gamma, *ck_gamma;
    const float *co_w, *co_b, *proj_w, *proj_b, *mlp0_w, *mlp0_b, *mlp2_w, *mlp2_b;
} p3d_block_weights;

/* io resblock weights (no reference): GN1 affine, conv1, GN2 affine, conv2. */
typedef struct p3d_resblock_weights {
    const float *gn1_w, *gn1_b, *conv1_w, *conv1_b, *gn2_w, *gn2_b, *conv2_w, *conv2_b;
} p3d_resblock_weights;

/* Model weights (SLatFlowWeightsF32, include/pixal3d/slat_flow.h:39-51),
 * f32 DEVICE pointers.  blocks: num_blocks entries; io_in/io_out:
 * io_resblocks entries each (may be NULL when io_resblocks == 0). */
typedef struct p3d_flow_weights {
    const float *input_w, *input_b, *t_w0, *t_b0, *t_w2, *t_b2, *mod_w, *mod_b, *output_w, *output_b;
    const p3d_block_weights *blocks;
    const p3d_resblock_weights *io_in, *io_out;
} p3d_flow_weights;

typedef struct p3d_flow p3d_flow;

/* Timestep conditioning of the flow model (timestep_embedding +
 * timestep_embed_mlp, src/flow.cpp:92-180, then SiLU and the adaLN
 * modulation linear, src/slat_flow.cpp:208-222): tmod[b] (6*channels) from
 * the model timestep timesteps[b].  f32 device weights: w0 [C][256], w2
 * [C][C], mod_w [6C][C].  scratch: batch * (256 + 2 * channels) floats. */
int p3d_timestep_mlp(p3d_ctx *ctx, const float *timesteps, int batch, int channels, const float *w0,
                     const float *b0, const float *w2, const float *b2, const float *mod_w, const float *mod_b,
                     float *scratch, float *tmod);

/* Upload/convert weights into the device layout (16-bit GEMM operands).
 * Replaces SLatFlowModel::load's tensor upload (src/slat_flow.cpp:578-663). */
int p3d_flow_create(p3d_ctx *ctx, const p3d_flow_hparams *hp, const p3d_flow_weights *w, p3d_flow **out);
int p3d_flow_destroy(p3d_flow *flow);

/* Bind a coordinate set (device coords [n][4], batch-contiguous, `batch`
 * items) and a condition layout (ctx_offsets[batch+1] host array) and size
 * workspaces.  Builds neighbour maps / downsample maps once. */
int p3d_flow_prepare(p3d_flow *flow, const int32_t *coords, int64_t n, int batch, int sx, int sy, int sz,
                     const int64_t *ctx_offsets_host);

/* One forward (slat_flow_forward_f32, src/slat_flow.cpp:161-249):
 * x f32 [n][in], timesteps f32 [batch] (device), ctx bf16 or f32
 * [T][cond] (ctx_dtype: P3D_F32, or the model's operand dtype), proj f32
 * [n][proj_in] or NULL, out f32 [n][out].  With a concat condition, x is
 * the caller's [input | concat] rows (concat_sparse_features, :50-75). */
int p3d_flow_forward(p3d_flow *flow, const float *x, const float *timesteps, const void *ctx_feats,
                     int ctx_dtype, const float *proj, float *out);

/* Sampler config (FlowEulerSamplerConfig, include/pixal3d/flow_sampler.h:14-23). */
typedef struct p3d_sampler_config {
    int steps;
    float sigma_min, rescale_t, guidance_strength, guidance_rescale;
    float guidance_interval_min, guidance_interval_max;
    int use_graph; /* capture one step as a CUDA graph and replay it */
} p3d_sampler_config;

/* SLatFlowModel::sample (src/slat_flow.cpp:1401-1447) with flow_euler_sample_f32
 * (src/flow_sampler.cpp:245-343) entirely on device.  The flow must have been
 * prepared with batch = 2*images: image i appears as batch item i
 * (conditional) and again as item images + i (unconditional, zeros
 * condition), with the same coordinates; rows contiguous per item.  ctx
 * layout: conditional tokens of image i in item i; items images.. are
 * cleared to zeros.  proj (proj mode): f32 [n/2][proj_in] for the
 * conditional rows (the unconditional copy uses zeros).  x: f32 [n/2][in],
 * the conditional rows, in/out. */
int p3d_flow_sample(p3d_flow *flow, float *x, const void *ctx_feats, int ctx_dtype, const float *proj,
                    const p3d_sampler_config *cfg);
/* The same with a concat condition (the texture stage's normalized shape
 * latent, src/slat_flow.cpp:1407-1447 and :171-181): the model input of
 * every forward, conditional and unconditional, is [state | concat] with
 * concat f32 [n/2][concat_channels] for the conditional rows; the model's
 * in_channels = out_channels + concat_channels; x holds the out_channels
 * state columns.  concat NULL with concat_channels 0 is p3d_flow_sample. */
int p3d_flow_sample_concat(p3d_flow *flow, float *x, const void *ctx_feats, int ctx_dtype, const float *proj,
                           const float *concat, int concat_channels, const p3d_sampler_config *cfg);
/* Kernel launches one sampler step issued (forward + update), for reporting. */
int64_t p3d_flow_launches_per_step(const p3d_flow *flow);

/* ------------------------------------------------------- SLat decoder */

#define P3D_DECODER_MAX_LEVELS 8

/* SLatDecoderConfig (include/pixal3d/slat_decoder.h): levels of
 * model_channels / num_blocks ConvNeXt blocks, a channel-to-spatial
 * res block between consecutive levels. */
typedef struct p3d_decoder_config {
    int latent_channels, out_channels, levels;
    int model_channels[P3D_DECODER_MAX_LEVELS];
    int num_blocks[P3D_DECODER_MAX_LEVELS];
    int pred_subdiv;
    float norm_eps;
    int operand_dtype; /* P3D_F16 or P3D_BF16 */
} p3d_decoder_config;

/* SLatDecoderBlockWeightsF32 (include/pixal3d/slat_decoder.h), f32 DEVICE
 * pointers.  kind 0 = ConvNeXt (norm, conv1, mlp0, mlp2), 1 =
 * channel-to-spatial res block (norm1, conv1, conv2, to_subdiv).  Conv
 * weights [27][cout][cin]. */
typedef struct p3d_decoder_block {
    int kind, channels, out_channels, mlp_hidden;
    const float *norm_w, *norm_b, *norm1_w, *norm1_b, *conv1_w, *conv1_b, *conv2_w, *conv2_b;
    const float *mlp0_w, *mlp0_b, *mlp2_w, *mlp2_b, *subdiv_w, *subdiv_b;
} p3d_decoder_block;

typedef struct p3d_decoder_weights {
    const float *from_latent_w, *from_latent_b, *output_w, *output_b;
    const p3d_decoder_block *blocks;
    int num_blocks;
} p3d_decoder_weights;

typedef struct p3d_decoder p3d_decoder;

/* Upload/convert the decoder weights into the device layout (16-bit,
 * padded operands).  Replaces SLatDecoderModel::load's tensor upload. */
int p3d_decoder_create(p3d_ctx *ctx, const p3d_decoder_config *cfg, const p3d_decoder_weights *w, p3d_decoder **out);
int p3d_decoder_destroy(p3d_decoder *dec);

/* slat_decoder_forward_f32 (src/slat_decoder.cpp:290-376) on the device, or
 * with stop_level in [0, levels) slat_decoder_upsample_coords_f32
 * (:378-455): stop at that level's input.  coords int32 [n][4] and latent
 * f32 [n][latent_channels] on the device.  guides: NULL or levels-1 device
 * pointers to f32 [rows(level)][8] subdivision logits (child c kept where
 * > 0) used when pred_subdiv is 0, with their row counts in guide_rows.
 * Synchronises once per level (the next level's size).  Results stay in the
 * decoder until the next run; read them with the calls below. */
int p3d_decoder_run(p3d_decoder *dec, const int32_t *coords, int64_t n, int batch, int sx, int sy, int sz,
                    const float *latent, const float *const *guides, const int64_t *guide_rows, int stop_level);
/* Rows of level l (l < levels; the output has the last level's rows). */
int64_t p3d_decoder_rows(const p3d_decoder *dec, int level);
/* Coordinates of level l -> out int32 [rows(l)][4] (device). */
int p3d_decoder_coords(p3d_decoder *dec, int level, int32_t *out);
/* Output features f32 [rows][out_channels] (device); after a stopped run,
 * the hidden features f32 [rows(stop)][model_channels[stop]]. */
int p3d_decoder_output(p3d_decoder *dec, float *out);
/* Predicted subdivision logits of level l (pred_subdiv), f32 [rows(l)][8]. */
int p3d_decoder_subdivision(p3d_decoder *dec, int level, float *out);

#ifdef __cplusplus
}
#endif

#endif /* P3D_H */
