// Shifted-window sparse self-attention (no reference implementation: the
// config-3 SLat decoder's 12 blocks of 8^3-window attention).
//
// Partition: row i with coords (b, x, y, z) belongs to window
//   (b, (x + shift) / W, (y + shift) / W, (z + shift) / W)
// on a grid of nw_d = ceil((s_d + shift) / W) windows per axis, window index
//   w = ((b * nwx + wx) * nwy + wy) * nwz + wz,  num_windows = batch * nwx * nwy * nwz.
// Two rows attend to each other iff they share a window; a shift of W/2 on
// alternate blocks moves the window boundaries (the Swin scheme).  The
// partition is a permutation perm (rows in window order; within a window by
// ascending row index, so the result is deterministic) and cu[w] = first
// position of window w, cu[num_windows] = n.  Empty windows have
// cu[w] == cu[w+1].
//
// Steps (all on the device, nothing read back):
//   1. key[i] = w(i), count[w] += 1                     (atomics)
//   2. cu = exclusive scan of count                    (one block)
//   3. perm[cu[w] + atomicAdd(cursor[w], 1)] = i       (atomics, any order)
//   4. each window's segment sorted ascending in shared memory (one block per
//      window, bitonic sort of <= 1024 entries)
// The attention gathers q/k/v rows into window order, runs the varlen
// tcgen05 attention with cu as both query and key offsets, and scatters the
// output rows back to the canonical order.
#include "p3d_common.cuh"

int p3d_fmha_tc(p3d_ctx *ctx, const void *q, int64_t ldq, const void *k, int64_t ldk, const void *v, int64_t ldv,
                void *out, int64_t ldo, const int32_t *cu_q, const int32_t *cu_k, int nseq, int64_t max_q,
                int64_t rows_q, int64_t rows_k, int heads, float scale, int dtype);

namespace p3d {
namespace {

constexpr int kMaxWindowRows = 1024;  // window^3 bound of the in-block sort

// A row outside [0, batch) x grid latches P3D_ERR_INVALID and is left out of
// every window (its key is -1).
__global__ void window_key_kernel(const int32_t *__restrict__ coords, int64_t n, int batch, int window, int shift,
                                  int sx, int sy, int sz, int nwx, int nwy, int nwz, int32_t *__restrict__ key,
                                  int32_t *__restrict__ count, int *fault) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = reinterpret_cast<const int4 *>(coords)[i];
    if (c.x < 0 || c.x >= batch || c.y < 0 || c.y >= sx || c.z < 0 || c.z >= sy || c.w < 0 || c.w >= sz) {
        key[i] = -1;
        latch_fault(fault, P3D_ERR_INVALID);
        return;
    }
    const int wx = (c.y + shift) / window, wy = (c.z + shift) / window, wz = (c.w + shift) / window;
    const int w = ((c.x * nwx + wx) * nwy + wy) * nwz + wz;
    key[i] = w;
    atomicAdd(count + w, 1);
}

// Exclusive scan of count[0..m) into cu[0..m], cu[m] = total; one block of
// 1024 threads walking the array in chunks (m is a few thousand windows).
__global__ void __launch_bounds__(1024) window_scan_kernel(const int32_t *__restrict__ count, int64_t m,
                                                           int32_t *__restrict__ cu) {
    __shared__ int32_t warp_sum[32];
    __shared__ int32_t carry_s;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    if (t == 0) carry_s = 0;
    __syncthreads();
    for (int64_t base = 0; base < m; base += 1024) {
        const int64_t i = base + t;
        const int32_t v = i < m ? count[i] : 0;
        int32_t x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_sum[warp] = x;
        __syncthreads();
        if (warp == 0) {
            int32_t s = warp_sum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int32_t y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += y;
            }
            warp_sum[lane] = s;  // inclusive over warps
        }
        __syncthreads();
        const int32_t carry = carry_s;
        const int32_t before = (warp > 0 ? warp_sum[warp - 1] : 0) + x - v;
        if (i < m) cu[i] = carry + before;
        __syncthreads();
        if (t == 0) carry_s = carry + warp_sum[31];
        __syncthreads();
    }
    if (t == 0) cu[m] = carry_s;
}

__global__ void window_fill_kernel(const int32_t *__restrict__ key, int64_t n, const int32_t *__restrict__ cu,
                                   int32_t *__restrict__ cursor, int32_t *__restrict__ perm) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int w = key[i];
    if (w >= 0) perm[cu[w] + atomicAdd(cursor + w, 1)] = static_cast<int32_t>(i);
}

// Bitonic sort of one window's segment (<= kMaxWindowRows entries) in shared
// memory, padded with INT32_MAX.
__global__ void __launch_bounds__(512) window_sort_kernel(const int32_t *__restrict__ cu, int32_t *__restrict__ perm) {
    __shared__ int32_t s[kMaxWindowRows];
    const int w = blockIdx.x;
    const int32_t b0 = cu[w], len = cu[w + 1] - b0;
    if (len <= 1) return;
    int size = 1;
    while (size < len) size <<= 1;
    for (int i = threadIdx.x; i < size; i += blockDim.x) s[i] = i < len ? perm[b0 + i] : 0x7fffffff;
    __syncthreads();
    for (int k = 2; k <= size; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < size; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const bool up = (i & k) == 0;
                    const int32_t a = s[i], b = s[ixj];
                    if ((a > b) == up) {
                        s[i] = b;
                        s[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < len; i += blockDim.x) perm[b0 + i] = s[i];
}

// dst[j] = src[rows[j]] (gather, scatter = 0) or dst[rows[j]] = src[j]
// (scatter = 1) for 16-bit rows of `cols` elements (cols % 8 == 0): one warp
// per row, 16-byte copies.
__global__ void permute_rows16_kernel(const uint16_t *__restrict__ src, int64_t lds, const int32_t *__restrict__ rows,
                                      int64_t n, int cols, uint16_t *__restrict__ dst, int64_t ldd, int scatter) {
    const int64_t j = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (j >= n) return;
    const int lane = threadIdx.x & 31;
    const int64_t r = rows[j];
    if (r < 0 || r >= n) return;  // position left empty by an invalid row
    const uint4 *s = reinterpret_cast<const uint4 *>(src + (scatter ? j : r) * lds);
    uint4 *d = reinterpret_cast<uint4 *>(dst + (scatter ? r : j) * ldd);
    for (int c = lane; c < cols / 8; c += 32) d[c] = s[c];
}

int permute_rows16(p3d_ctx *ctx, const void *src, int64_t lds, const int32_t *rows, int64_t n, int cols, void *dst,
                   int64_t ldd, int scatter) {
    if (n == 0) return P3D_OK;
    permute_rows16_kernel<<<static_cast<unsigned>(ceil_div(n, 8)), 256, 0, ctx->stream>>>(
        static_cast<const uint16_t *>(src), lds, rows, n, cols, static_cast<uint16_t *>(dst), ldd, scatter);
    return check_launch(ctx, "permute_rows16");
}

}  // namespace
}  // namespace p3d

using namespace p3d;

extern "C" int64_t p3d_window_count(int batch, int window, int shift, int sx, int sy, int sz) {
    if (batch <= 0 || window <= 0 || shift < 0 || sx <= 0 || sy <= 0 || sz <= 0) return 0;
    const int64_t nx = (sx + shift + window - 1) / window, ny = (sy + shift + window - 1) / window,
                  nz = (sz + shift + window - 1) / window;
    return static_cast<int64_t>(batch) * nx * ny * nz;
}

extern "C" size_t p3d_window_partition_workspace(int64_t n, int64_t num_windows) {
    auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
    return up(sizeof(int32_t) * static_cast<size_t>(n)) + 2 * up(sizeof(int32_t) * static_cast<size_t>(num_windows));
}

extern "C" int p3d_window_partition(p3d_ctx *ctx, const int32_t *coords, int64_t n, int batch, int window, int shift,
                                    int sx, int sy, int sz, int32_t *perm, int32_t *cu, void *ws, size_t ws_bytes) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, coords && perm && cu && ws, "p3d_window_partition: null pointer");
    P3D_REQUIRE(ctx, (reinterpret_cast<uintptr_t>(coords) & 15) == 0, "p3d_window_partition: coords must be 16-byte aligned");
    P3D_REQUIRE(ctx, window > 0 && static_cast<int64_t>(window) * window * window <= kMaxWindowRows,
                "p3d_window_partition: window^3 must be at most 1024 rows");
    P3D_REQUIRE(ctx, shift >= 0 && shift < window, "p3d_window_partition: shift must be in [0, window)");
    P3D_REQUIRE(ctx, n >= 0 && n < (int64_t(1) << 31), "p3d_window_partition: bad n");
    const int64_t m = p3d_window_count(batch, window, shift, sx, sy, sz);
    P3D_REQUIRE(ctx, m > 0 && m < (int64_t(1) << 31), "p3d_window_partition: bad batch or grid");
    P3D_REQUIRE(ctx, ws_bytes >= p3d_window_partition_workspace(n, m), "p3d_window_partition: workspace too small");
    DeviceGuard guard(ctx->device);
    auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
    uint8_t *base = static_cast<uint8_t *>(ws);
    int32_t *key = reinterpret_cast<int32_t *>(base);
    int32_t *count = reinterpret_cast<int32_t *>(base + up(sizeof(int32_t) * n));
    int32_t *cursor = reinterpret_cast<int32_t *>(base + up(sizeof(int32_t) * n) + up(sizeof(int32_t) * m));
    P3D_CUDA(ctx, cudaMemsetAsync(count, 0, sizeof(int32_t) * m, ctx->stream));
    P3D_CUDA(ctx, cudaMemsetAsync(cursor, 0, sizeof(int32_t) * m, ctx->stream));
    P3D_CUDA(ctx, cudaMemsetAsync(perm, 0xff, sizeof(int32_t) * n, ctx->stream));  // -1: no row
    const int nwx = static_cast<int>((sx + shift + window - 1) / window);
    const int nwy = static_cast<int>((sy + shift + window - 1) / window);
    const int nwz = static_cast<int>((sz + shift + window - 1) / window);
    if (n > 0) {
        window_key_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, ctx->stream>>>(
            coords, n, batch, window, shift, sx, sy, sz, nwx, nwy, nwz, key, count, ctx->fault);
        int rc = check_launch(ctx, "window_key");
        if (rc) return rc;
    }
    window_scan_kernel<<<1, 1024, 0, ctx->stream>>>(count, m, cu);
    int rc = check_launch(ctx, "window_scan");
    if (rc || n == 0) return rc;
    window_fill_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, ctx->stream>>>(key, n, cu, cursor, perm);
    if ((rc = check_launch(ctx, "window_fill"))) return rc;
    window_sort_kernel<<<static_cast<unsigned>(m), 512, 0, ctx->stream>>>(cu, perm);
    return check_launch(ctx, "window_sort");
}

extern "C" size_t p3d_window_attention_scratch(int64_t n, int heads) {
    return 4 * static_cast<size_t>(n) * static_cast<size_t>(heads) * 64 * sizeof(uint16_t);
}

extern "C" int p3d_window_attention(p3d_ctx *ctx, const void *q, int64_t ldq, const void *k, int64_t ldk,
                                    const void *v, int64_t ldv, const int32_t *perm, const int32_t *cu,
                                    int64_t num_windows, int max_window_rows, int64_t n, int heads, int head_dim,
                                    float scale, int dtype, void *scratch, size_t scratch_bytes, void *out,
                                    int64_t ldo) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, q && k && v && perm && cu && scratch && out, "p3d_window_attention: null pointer");
    P3D_REQUIRE(ctx, head_dim == 64, "p3d_window_attention: head_dim must be 64");
    P3D_REQUIRE(ctx, is_16bit(dtype), "p3d_window_attention: dtype must be bf16 or f16");
    P3D_REQUIRE(ctx, heads > 0 && heads < 65536, "p3d_window_attention: bad heads");
    P3D_REQUIRE(ctx, num_windows > 0 && num_windows < 65536, "p3d_window_attention: 1..65535 windows");
    P3D_REQUIRE(ctx, max_window_rows > 0, "p3d_window_attention: bad window row bound");
    P3D_REQUIRE(ctx, scale > 0.0f, "p3d_window_attention: scale must be positive");
    P3D_REQUIRE(ctx, ldq % 8 == 0 && ldk % 8 == 0 && ldv % 8 == 0 && ldo % 8 == 0,
                "p3d_window_attention: leading dimensions must keep 16-byte rows");
    P3D_REQUIRE(ctx,
                ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
                  reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(scratch)) & 15) == 0,
                "p3d_window_attention: q/k/v/out/scratch must be 16-byte aligned");
    P3D_REQUIRE(ctx, n >= 0 && n < (int64_t(1) << 31), "p3d_window_attention: bad n");
    P3D_REQUIRE(ctx, scratch_bytes >= p3d_window_attention_scratch(n, heads),
                "p3d_window_attention: scratch too small");
    if (n == 0) return P3D_OK;
    DeviceGuard guard(ctx->device);
    const int cols = heads * 64;
    uint16_t *wq = static_cast<uint16_t *>(scratch);
    uint16_t *wk = wq + n * cols;
    uint16_t *wv = wk + n * cols;
    uint16_t *wo = wv + n * cols;
    int rc;
    if ((rc = permute_rows16(ctx, q, ldq, perm, n, cols, wq, cols, 0))) return rc;
    if ((rc = permute_rows16(ctx, k, ldk, perm, n, cols, wk, cols, 0))) return rc;
    if ((rc = permute_rows16(ctx, v, ldv, perm, n, cols, wv, cols, 0))) return rc;
    if ((rc = p3d_fmha_tc(ctx, wq, cols, wk, cols, wv, cols, wo, cols, cu, cu, static_cast<int>(num_windows),
                          max_window_rows, n, n, heads, scale, dtype)))
        return rc;
    return permute_rows16(ctx, wo, cols, perm, n, cols, out, ldo, 1);
}
