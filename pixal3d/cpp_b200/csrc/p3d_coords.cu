// Integer/topology kernels: coordinate hash, 27-offset neighbour maps,
// downsample (mean pool) topology, nearest upsample, channel-to-spatial
// (subdivide) topology and feature gathers.
//
// All of it is integer-exact: the neighbour map, the downsampled coordinate
// order and the subdivided coordinate order are bit-identical to the
// reference (src/slat_decoder.cpp:670-714, src/sparse.cpp:536-702).
#include <cub/device/device_radix_sort.cuh>

#include "p3d_common.cuh"

namespace p3d {
namespace {

constexpr uint64_t kEmpty = ~0ull;
constexpr int kMaxProbes = 1 << 16;

// A key holds 16 bits per field: batch in [0, 65536), x/y/z in [-32768,
// 32768).  Coordinates outside that range would alias another key, so the
// hash build refuses them (P3D_ERR_INVALID) and lookups of such a neighbour
// report it missing.
__device__ __forceinline__ bool key_packable(int b, int x, int y, int z) {
    return static_cast<unsigned>(b) < 65536u && static_cast<unsigned>(x + 32768) < 65536u &&
           static_cast<unsigned>(y + 32768) < 65536u && static_cast<unsigned>(z + 32768) < 65536u;
}

__device__ __forceinline__ uint64_t pack_key(int b, int x, int y, int z) {
    return (static_cast<uint64_t>(static_cast<uint32_t>(b) & 0xFFFFu) << 48) |
           (static_cast<uint64_t>(static_cast<uint32_t>(x + 32768) & 0xFFFFu) << 32) |
           (static_cast<uint64_t>(static_cast<uint32_t>(y + 32768) & 0xFFFFu) << 16) |
           static_cast<uint64_t>(static_cast<uint32_t>(z + 32768) & 0xFFFFu);
}

__device__ __forceinline__ uint64_t mix64(uint64_t k) {
    k ^= k >> 33;
    k *= 0xff51afd7ed558ccdull;
    k ^= k >> 33;
    k *= 0xc4ceb9fe1a85ec53ull;
    k ^= k >> 33;
    return k;
}

__global__ void fill_u64_kernel(uint64_t *p, int64_t n, uint64_t v) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

__global__ void fill_i32_kernel(int32_t *p, int64_t n, int32_t v) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

// Bucketed linear probing, warp-cooperative: the table is read in windows of
// kTile = 4 consecutive slots (32 bytes of keys, one L2 sector), starting at
// the key's home window and moving to the next window while the current one
// is full.  A 4-lane tile of a warp handles one key: each lane reads one slot
// of the window, ballots tell the tile where the key and the empty slots are,
// and the lowest empty slot is claimed by CAS.  (4-lane tiles measured
// faster than 8-lane ones: a 43,532-point map 52 vs 70 us, 884,736 points
// 0.69 vs 1.08 ms; the lookups are bound by instruction issue, which the
// lanes per key multiply.)  A key therefore sits behind no
// empty slot of its probe sequence, so a scalar scan from the home window
// (hash_find) and the cooperative scan (tile_find) agree.
constexpr int kTile = 4;
constexpr int kMaxWindows = kMaxProbes / kTile;

__device__ __forceinline__ uint64_t home_slot(uint64_t key, uint64_t mask) {
    return (mix64(key) & mask) & ~static_cast<uint64_t>(kTile - 1);
}

// Thread t of the grid is lane (t % kTile) of the tile of key t / kTile (a
// tile never straddles a warp; the grid has kTile n threads, so whole tiles
// exit together).
__global__ void hash_insert_kernel(const int4 *__restrict__ coords, int64_t n, uint64_t *keys, int32_t *vals,
                                   uint64_t mask, int *fault) {
    const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kTile;
    if (i >= n) return;
    const int lane = threadIdx.x & 31, l = lane & (kTile - 1);
    const unsigned tmask = ((1u << kTile) - 1u) << (lane & ~(kTile - 1));
    const int4 c = coords[i];
    if (!key_packable(c.x, c.y, c.z, c.w)) {
        if (l == 0) latch_fault(fault, P3D_ERR_INVALID);
        return;
    }
    const uint64_t key = pack_key(c.x, c.y, c.z, c.w);
    uint64_t base = home_slot(key, mask);
    for (int w = 0; w < kMaxWindows; ++w) {
        const uint64_t slot = base + l;
        const uint64_t k = *reinterpret_cast<volatile const uint64_t *>(keys + slot);
        if (__ballot_sync(tmask, k == key)) {
            if (l == 0) latch_fault(fault, P3D_ERR_DUPLICATE);
            return;
        }
        unsigned empty = __ballot_sync(tmask, k == kEmpty);
        while (empty) {
            const int leader = __ffs(empty) - 1;
            unsigned long long prev = 0;
            if (lane == leader)
                prev = atomicCAS(reinterpret_cast<unsigned long long *>(keys + slot), kEmpty,
                                 static_cast<unsigned long long>(key));
            prev = __shfl_sync(tmask, prev, leader);
            if (prev == kEmpty) {
                if (lane == leader) vals[slot] = static_cast<int32_t>(i);
                return;
            }
            if (prev == key) {
                if (lane == leader) latch_fault(fault, P3D_ERR_DUPLICATE);
                return;
            }
            empty &= ~(1u << leader);  // taken by another key meanwhile: next empty slot of the window
        }
        base = (base + kTile) & mask;
    }
    if (l == 0) latch_fault(fault, P3D_ERR_HASH_FULL);
}

// Validation insert: every row inserts its key; the slot's value ends as the
// smallest row index holding that key (vals pre-filled with INT32_MAX).
__global__ void validate_insert_kernel(const int4 *__restrict__ coords, int64_t n, uint64_t *keys, int32_t *vals,
                                       uint64_t mask, int *fault) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = coords[i];
    if (!key_packable(c.x, c.y, c.z, c.w)) return;  // outside every accepted shape: reported as a bounds error
    const uint64_t key = pack_key(c.x, c.y, c.z, c.w);
    uint64_t slot = home_slot(key, mask);
    for (int probe = 0; probe < kMaxProbes; ++probe) {
        const unsigned long long prev =
            atomicCAS(reinterpret_cast<unsigned long long *>(keys + slot), kEmpty, static_cast<unsigned long long>(key));
        if (prev == kEmpty || prev == key) {
            atomicMin(vals + slot, static_cast<int32_t>(i));
            return;
        }
        slot = (slot + 1) & mask;
    }
    latch_fault(fault, P3D_ERR_HASH_FULL);
}

__device__ __forceinline__ int32_t hash_find(const uint64_t *__restrict__ keys, const int32_t *__restrict__ vals,
                                             uint64_t mask, uint64_t key, int32_t miss) {
    uint64_t slot = home_slot(key, mask);
    for (int probe = 0; probe < kMaxProbes; ++probe) {
        const uint64_t k = __ldg(reinterpret_cast<const unsigned long long *>(keys + slot));
        if (k == key) return __ldg(vals + slot);
        if (k == kEmpty) return miss;
        slot = (slot + 1) & mask;
    }
    return miss;
}

// Cooperative lookup by the kTile-lane tile of the calling lane (all lanes of
// the tile pass the same key); every lane returns the row or `miss`.
__device__ __forceinline__ int32_t tile_find(const uint64_t *__restrict__ keys, const int32_t *__restrict__ vals,
                                             uint64_t mask, uint64_t key, int32_t miss, unsigned tmask, int l) {
    uint64_t base = home_slot(key, mask);
    for (int w = 0; w < kMaxWindows; ++w) {
        const uint64_t k = __ldg(reinterpret_cast<const unsigned long long *>(keys + base + l));
        const unsigned hit = __ballot_sync(tmask, k == key);
        if (hit) {
            const int32_t v = k == key ? __ldg(vals + base + l) : 0;
            return __shfl_sync(tmask, v, __ffs(hit) - 1);
        }
        if (__ballot_sync(tmask, k == kEmpty)) return miss;
        base = (base + kTile) & mask;
    }
    return miss;
}

// Tile per (tap, point): nbr[tap*n + p] = row of (b, x+kd-1, y+kh-1, z+kw-1) or n.
__global__ void neighbor_map_kernel(const int4 *__restrict__ coords, int64_t n, const uint64_t *__restrict__ keys,
                                    const int32_t *__restrict__ vals, uint64_t mask, int32_t *__restrict__ nbr) {
    const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kTile;
    if (i >= 27 * n) return;
    const int lane = threadIdx.x & 31, l = lane & (kTile - 1);
    const unsigned tmask = ((1u << kTile) - 1u) << (lane & ~(kTile - 1));
    const int tap = static_cast<int>(i / n);
    const int64_t p = i - static_cast<int64_t>(tap) * n;
    const int kd = tap / 9, kh = (tap / 3) % 3, kw = tap % 3;
    const int4 c = __ldg(coords + p);
    const int x = c.y + kd - 1, y = c.z + kh - 1, z = c.w + kw - 1;
    int32_t r = static_cast<int32_t>(n);
    if (key_packable(c.x, x, y, z)) r = tile_find(keys, vals, mask, pack_key(c.x, x, y, z), r, tmask, l);
    if (l == 0) nbr[i] = r;
}

// ------------------------------------------------------------------ scans
// Exclusive int32 scan in three launches: per-block totals, a single-block
// scan of the totals, then per-block scans with the block offset.
constexpr int kScanBlock = 1024;

__device__ __forceinline__ int block_exclusive_scan(int v, int *warp_sums, int &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int s = lane < (blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        warp_sums[lane] = s;
    }
    __syncthreads();
    const int prefix = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
    total = warp_sums[(blockDim.x >> 5) - 1];
    __syncthreads();
    return prefix;
}

__global__ void scan_block_totals(const int32_t *__restrict__ in, int64_t n, int32_t *__restrict__ totals) {
    __shared__ int ws[32];
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kScanBlock + threadIdx.x;
    int total;
    block_exclusive_scan(i < n ? in[i] : 0, ws, total);
    if (threadIdx.x == 0) totals[blockIdx.x] = total;
}

__global__ void scan_totals_single(int32_t *totals, int64_t nb, int32_t *grand_total) {
    __shared__ int ws[32];
    int carry = 0;
    for (int64_t base = 0; base < nb; base += kScanBlock) {
        const int64_t i = base + threadIdx.x;
        const int v = i < nb ? totals[i] : 0;
        int total;
        const int ex = block_exclusive_scan(v, ws, total);
        if (i < nb) totals[i] = ex + carry;
        carry += total;
    }
    if (threadIdx.x == 0 && grand_total) *grand_total = carry;
}

__global__ void scan_apply(const int32_t *__restrict__ in, int64_t n, const int32_t *__restrict__ totals,
                           int32_t *__restrict__ out) {
    __shared__ int ws[32];
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kScanBlock + threadIdx.x;
    int total;
    const int v = i < n ? in[i] : 0;
    const int ex = block_exclusive_scan(v, ws, total);
    if (i < n) out[i] = ex + totals[blockIdx.x];
}

// in/out may alias.  scratch: ceil(n/1024) + 1 int32.  grand_total: device int32.
int exclusive_scan(p3d_ctx *ctx, const int32_t *in, int64_t n, int32_t *out, int32_t *scratch, int32_t *grand_total) {
    const int64_t nb = ceil_div(n, kScanBlock);
    if (nb == 0) {  // empty input: only publish a zero total
        scan_totals_single<<<1, kScanBlock, 0, ctx->stream>>>(scratch, 0, grand_total);
        return check_launch(ctx, "scan_totals_single");
    }
    scan_block_totals<<<static_cast<unsigned>(nb), kScanBlock, 0, ctx->stream>>>(in, n, scratch);
    int rc = check_launch(ctx, "scan_block_totals");
    if (rc) return rc;
    scan_totals_single<<<1, kScanBlock, 0, ctx->stream>>>(scratch, nb, grand_total);
    rc = check_launch(ctx, "scan_totals_single");
    if (rc) return rc;
    scan_apply<<<static_cast<unsigned>(nb), kScanBlock, 0, ctx->stream>>>(in, n, scratch, out);
    return check_launch(ctx, "scan_apply");
}

// ------------------------------------------------------------ downsample
__global__ void down_mark_kernel(const int4 *__restrict__ coords, int64_t n, int batch, int sx, int sy, int sz, int f,
                                 int gx, int gy, int gz, int32_t *grid, int *fault) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = coords[i];
    if (c.x < 0 || c.x >= batch || c.y < 0 || c.y >= sx || c.z < 0 || c.z >= sy || c.w < 0 || c.w >= sz) {
        latch_fault(fault, P3D_ERR_INVALID);
        return;
    }
    const int64_t cell = ((static_cast<int64_t>(c.x) * gx + c.y / f) * gy + c.z / f) * gz + c.w / f;
    grid[cell] = 1;
}

__global__ void down_assign_kernel(const int4 *__restrict__ coords, int64_t n, int batch, int sx, int sy, int sz,
                                   int f, int gx, int gy, int gz, const int32_t *__restrict__ rank, int32_t *parent,
                                   int32_t *child, int4 *out_coords) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = coords[i];
    // Rows outside the shape were latched as invalid by down_mark_kernel;
    // skip them here so no grid cell outside [0, cells) is read.
    if (c.x < 0 || c.x >= batch || c.y < 0 || c.y >= sx || c.z < 0 || c.z >= sy || c.w < 0 || c.w >= sz) {
        parent[i] = -1;
        return;
    }
    const int px = c.y / f, py = c.z / f, pz = c.w / f;
    const int64_t cell = ((static_cast<int64_t>(c.x) * gx + px) * gy + py) * gz + pz;
    const int32_t p = rank[cell];
    parent[i] = p;
    const int oct = ((c.y % f) * f + (c.z % f)) * f + (c.w % f);
    child[static_cast<int64_t>(p) * f * f * f + oct] = static_cast<int32_t>(i);
    out_coords[p] = make_int4(c.x, px, py, pz);
}

__global__ void i32_to_i64_kernel(const int32_t *src, int64_t *dst) { *dst = *src; }

// Mean over children in octant order; one warp per output row.
template <typename T>
__global__ void down_mean_kernel(const T *__restrict__ x, int64_t m, int channels, int nchild,
                                 const int32_t *__restrict__ child, T *__restrict__ out) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= m) return;
    const int lane = threadIdx.x & 31;
    const int32_t *ch = child + row * nchild;
    for (int c = lane; c < channels; c += 32) {
        float s = 0.0f;
        int cnt = 0;
        for (int o = 0; o < nchild; ++o) {
            const int32_t src = __ldg(ch + o);
            if (src >= 0) {
                s += to_f32(x[static_cast<int64_t>(src) * channels + c]);
                ++cnt;
            }
        }
        const float v = cnt ? s / static_cast<float>(cnt) : 0.0f;
        out[row * channels + c] = from_f32<T>(v);
    }
}

// f32 rows, 8 children, channels % 4 == 0: one warp per parent row, float4
// per lane, the 8 children's loads issued before the sums (added in child
// order, as the scalar kernel does).
__global__ void down_mean8_f32_kernel(const float *__restrict__ x, int64_t m, int channels,
                                      const int32_t *__restrict__ child, float *__restrict__ out) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= m) return;
    const int lane = threadIdx.x & 31;
    int32_t src[8];
#pragma unroll
    for (int o = 0; o < 8; ++o) src[o] = __ldg(child + row * 8 + o);
    const int c4 = channels / 4;
    for (int c = lane; c < c4; c += 32) {
        float4 v[8];
#pragma unroll
        for (int o = 0; o < 8; ++o)
            v[o] = src[o] >= 0 ? __ldg(reinterpret_cast<const float4 *>(x + static_cast<int64_t>(src[o]) * channels) + c)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        int cnt = 0;
#pragma unroll
        for (int o = 0; o < 8; ++o) {
            if (src[o] >= 0) {
                s.x += v[o].x;
                s.y += v[o].y;
                s.z += v[o].z;
                s.w += v[o].w;
                ++cnt;
            }
        }
        const float inv = cnt ? static_cast<float>(cnt) : 1.0f;
        reinterpret_cast<float4 *>(out + row * channels)[c] =
            cnt ? make_float4(s.x / inv, s.y / inv, s.z / inv, s.w / inv) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

template <typename T>
__global__ void gather_rows_kernel(const T *__restrict__ x, int64_t n, int channels, const int32_t *__restrict__ idx,
                                   T *__restrict__ out) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n) return;
    const int lane = threadIdx.x & 31;
    const int64_t src = idx[row];
    for (int c = lane; c < channels; c += 32) out[row * channels + c] = x[src * channels + c];
}

// ---------------------------------------------------- channel-to-spatial
__global__ void c2s_count_kernel(int64_t n, int nchild, const float *__restrict__ mask, int32_t *counts) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int cnt = nchild;
    if (mask) {
        cnt = 0;
        for (int c = 0; c < nchild; ++c) cnt += mask[i * nchild + c] > 0.0f ? 1 : 0;
    }
    counts[i] = cnt;
}

__global__ void c2s_emit_kernel(const int4 *__restrict__ coords, int64_t n, int f, const float *__restrict__ mask,
                                const int32_t *__restrict__ offsets, int4 *out_coords, int32_t *src_row,
                                int8_t *src_child) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int nchild = f * f * f;
    const int4 c = coords[i];
    int64_t o = offsets[i];
    for (int ch = 0; ch < nchild; ++ch) {
        if (mask && !(mask[i * nchild + ch] > 0.0f)) continue;
        const int cx = ch % f, cy = (ch / f) % f, cz = ch / (f * f);
        out_coords[o] = make_int4(c.x, c.y * f + cx, c.z * f + cy, c.w * f + cz);
        src_row[o] = static_cast<int32_t>(i);
        src_child[o] = static_cast<int8_t>(ch);
        ++o;
    }
}

template <typename T>
__global__ void c2s_gather_kernel(const T *__restrict__ x, int64_t in_ch, const int32_t *__restrict__ src_row,
                                  const int8_t *__restrict__ src_child, int64_t m, int cout, int repeat,
                                  T *__restrict__ out) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= m) return;
    const int lane = threadIdx.x & 31;
    // the child's channel slice must lie inside the source row
    if ((static_cast<int64_t>(src_child[row]) + 1) * cout > in_ch || src_child[row] < 0) return;
    const T *src = x + static_cast<int64_t>(src_row[row]) * in_ch + static_cast<int64_t>(src_child[row]) * cout;
    const int oc = cout * repeat;
    for (int c = lane; c < oc; c += 32) out[row * oc + c] = src[c / repeat];
}

unsigned blocks_for(int64_t n, int threads) { return static_cast<unsigned>(ceil_div(n, threads)); }

// offsets[b] = first row whose batch index is >= b (binary search over the
// batch-contiguous coordinate list), offsets[batch] = n.
__global__ void batch_offsets_kernel(const int4 *__restrict__ coords, int64_t n, int batch, int32_t *__restrict__ off) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b > batch) return;
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (coords[mid].x < b) lo = mid + 1; else hi = mid;
    }
    off[b] = static_cast<int32_t>(b == batch ? n : lo);
}

// Sort key of a fine-level row: (batch, neighbour pattern), pattern bit t
// set when nbr[t][row] is a point.
__global__ void row_pattern_key_kernel(const int4 *__restrict__ coords, const int32_t *__restrict__ nbr, int64_t n,
                                       int64_t chunk_rows, int chunk_bits, uint64_t *__restrict__ keys,
                                       int32_t *__restrict__ idx) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t m = 0;
    for (int t = 0; t < 27; ++t) {
        const int32_t s = __ldg(nbr + static_cast<int64_t>(t) * n + i);
        if (s >= 0 && s < n) m |= 1u << t;
    }
    const uint64_t chunk = static_cast<uint64_t>(i / chunk_rows);
    keys[i] = (static_cast<uint64_t>(static_cast<uint32_t>(__ldg(&coords[i].x))) << (27 + chunk_bits)) | (chunk << 27) | m;
    idx[i] = static_cast<int32_t>(i);
}

int bits_for(int64_t count) {
    int bits = 0;
    while ((int64_t(1) << bits) < count) ++bits;
    return bits;
}

// chunk_rows normalised: <= 0 or >= n means one chunk
int64_t row_order_chunk(int64_t n, int64_t chunk_rows) { return chunk_rows <= 0 || chunk_rows >= n ? std::max<int64_t>(n, 1) : chunk_rows; }

int row_order_end_bit(int64_t n, int batch, int64_t chunk_rows) {
    const int64_t chunk = row_order_chunk(n, chunk_rows);
    return 27 + bits_for((n + chunk - 1) / chunk) + std::max(1, bits_for(batch));
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

size_t row_order_temp_bytes(int64_t n, int batch, int64_t chunk_rows) {
    size_t temp = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, temp, static_cast<const uint64_t *>(nullptr),
                                    static_cast<uint64_t *>(nullptr), static_cast<const int32_t *>(nullptr),
                                    static_cast<int32_t *>(nullptr), static_cast<int>(n), 0,
                                    row_order_end_bit(n, batch, chunk_rows));
    return temp;
}

}  // namespace
}  // namespace p3d

using namespace p3d;

extern "C" size_t p3d_conv_row_order_workspace(int64_t n, int batch, int64_t chunk_rows) {
    if (n < 0 || batch <= 0 || n >= (int64_t(1) << 31) || row_order_end_bit(n, batch, chunk_rows) > 64) return 0;
    return align256(sizeof(uint64_t) * n) * 2 + align256(sizeof(int32_t) * n) +
           align256(row_order_temp_bytes(n, batch, chunk_rows)) + 256;
}

extern "C" int p3d_conv_row_order(p3d_ctx *ctx, const int32_t *coords, const int32_t *nbr, int64_t n, int batch,
                                  int64_t chunk_rows, void *ws, size_t ws_bytes, int32_t *perm) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, coords && nbr && perm && ws && batch > 0 && n >= 0 && n < (int64_t(1) << 31),
                "p3d_conv_row_order: bad argument");
    P3D_REQUIRE(ctx, row_order_end_bit(n, batch, chunk_rows) <= 64,
                "p3d_conv_row_order: chunk_rows too small for a 64-bit (batch, chunk, pattern) key");
    P3D_REQUIRE(ctx, (reinterpret_cast<uintptr_t>(coords) & 15) == 0 && (reinterpret_cast<uintptr_t>(ws) & 255) == 0,
                "p3d_conv_row_order: coords must be 16-byte and ws 256-byte aligned");
    P3D_REQUIRE(ctx, ws_bytes >= p3d_conv_row_order_workspace(n, batch, chunk_rows),
                "p3d_conv_row_order: workspace too small");
    if (n == 0) return P3D_OK;
    uint8_t *w = static_cast<uint8_t *>(ws);
    uint64_t *keys_in = reinterpret_cast<uint64_t *>(w);
    uint64_t *keys_out = reinterpret_cast<uint64_t *>(w + align256(sizeof(uint64_t) * n));
    int32_t *idx = reinterpret_cast<int32_t *>(w + 2 * align256(sizeof(uint64_t) * n));
    void *temp = w + 2 * align256(sizeof(uint64_t) * n) + align256(sizeof(int32_t) * n);
    size_t temp_bytes = row_order_temp_bytes(n, batch, chunk_rows);
    const int64_t chunk = row_order_chunk(n, chunk_rows);
    row_pattern_key_kernel<<<blocks_for(n, 256), 256, 0, ctx->stream>>>(
        reinterpret_cast<const int4 *>(coords), nbr, n, chunk, bits_for((n + chunk - 1) / chunk), keys_in, idx);
    int rc = check_launch(ctx, "row_pattern_key");
    if (rc) return rc;
    const cudaError_t e = cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys_in, keys_out, idx, perm,
                                                          static_cast<int>(n), 0, row_order_end_bit(n, batch, chunk_rows),
                                                          ctx->stream);
    if (e != cudaSuccess) return set_error(ctx, P3D_ERR_CUDA, std::string("p3d_conv_row_order: ") + cudaGetErrorString(e));
    return check_launch(ctx, "row_order_sort");
}

extern "C" int64_t p3d_coord_hash_capacity(int64_t n) {
    int64_t cap = 64;
    while (cap < 2 * n) cap <<= 1;
    return cap;
}

extern "C" int p3d_coord_hash_build(p3d_ctx *ctx, const int32_t *coords, int64_t n, uint64_t *keys, int32_t *vals,
                                    int64_t capacity) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, coords && keys && vals, "p3d_coord_hash_build: null pointer");
    P3D_REQUIRE(ctx, capacity >= 64 && (capacity & (capacity - 1)) == 0 && capacity >= n,
                "p3d_coord_hash_build: capacity must be a power of two >= max(n, 64)");
    P3D_REQUIRE(ctx, n < (int64_t(1) << 31), "p3d_coord_hash_build: too many points");
    fill_u64_kernel<<<blocks_for(capacity, 256), 256, 0, ctx->stream>>>(keys, capacity, kEmpty);
    int rc = check_launch(ctx, "fill_u64");
    if (rc || n == 0) return rc;
    hash_insert_kernel<<<blocks_for(n * kTile, 256), 256, 0, ctx->stream>>>(reinterpret_cast<const int4 *>(coords), n, keys,
                                                                    vals, static_cast<uint64_t>(capacity - 1),
                                                                    ctx->fault);
    return check_launch(ctx, "hash_insert");
}

extern "C" int p3d_neighbor_map27(p3d_ctx *ctx, const int32_t *coords, int64_t n, const uint64_t *keys,
                                  const int32_t *vals, int64_t capacity, int32_t *nbr_out) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, coords && keys && vals && nbr_out, "p3d_neighbor_map27: null pointer");
    P3D_REQUIRE(ctx, capacity > 0 && (capacity & (capacity - 1)) == 0, "p3d_neighbor_map27: bad capacity");
    P3D_REQUIRE(ctx, n < (int64_t(1) << 31) / 27, "p3d_neighbor_map27: too many points");
    P3D_REQUIRE(ctx, capacity >= 64, "p3d_neighbor_map27: capacity below 64 slots");
    if (n == 0) return P3D_OK;
    neighbor_map_kernel<<<blocks_for(27 * n * kTile, 256), 256, 0, ctx->stream>>>(
        reinterpret_cast<const int4 *>(coords), n, keys, vals, static_cast<uint64_t>(capacity - 1), nbr_out);
    return check_launch(ctx, "neighbor_map");
}

extern "C" size_t p3d_neighbor_map27_workspace(int64_t n) {
    const int64_t cap = p3d_coord_hash_capacity(n);
    return static_cast<size_t>(cap) * 8 + static_cast<size_t>(cap) * 4 + 256;
}

namespace p3d {
namespace {
// Per row, the first failing check in the order SparseTensorF32::valid
// applies them (src/sparse.cpp:286-308): 0 outside the shape, 1 duplicate of
// an earlier row, 2 batch index decreasing; folded into *first as
// (row << 2 | code) by atomicMin, so *first ends as the reference's first
// error.  Finiteness (code 3) is folded in by validate_finite_kernel.
__global__ void validate_points_kernel(const int4 *__restrict__ coords, int64_t n, int batch, int sx, int sy, int sz,
                                       const uint64_t *__restrict__ keys, const int32_t *__restrict__ vals,
                                       uint64_t mask, unsigned long long *first) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = coords[i];
    int code = -1;
    if (c.x < 0 || c.x >= batch || c.y < 0 || c.y >= sx || c.z < 0 || c.z >= sy || c.w < 0 || c.w >= sz) {
        code = 0;
    } else if (hash_find(keys, vals, mask, pack_key(c.x, c.y, c.z, c.w), -1) != static_cast<int32_t>(i)) {
        code = 1;
    } else if (i > 0 && coords[i - 1].x > c.x) {
        code = 2;
    }
    if (code >= 0) atomicMin(first, (static_cast<unsigned long long>(i) << 2) | static_cast<unsigned long long>(code));
}

__global__ void validate_finite_kernel(const float *__restrict__ x, int64_t count, int channels,
                                       unsigned long long *first) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= count) return;
    if (!isfinite(x[e])) atomicMin(first, (static_cast<unsigned long long>(e / channels) << 2) | 3ull);
}
}  // namespace
}  // namespace p3d

extern "C" size_t p3d_sparse_validate_workspace(int64_t n) { return p3d_neighbor_map27_workspace(n); }

extern "C" int p3d_sparse_validate(p3d_ctx *ctx, const int32_t *coords, int64_t n, const float *feats, int channels,
                                   int batch, int sx, int sy, int sz, void *ws, size_t ws_bytes, int64_t *first_bad) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, first_bad && n >= 0 && channels > 0, "p3d_sparse_validate: bad argument");
    P3D_REQUIRE(ctx, !feats || n < (int64_t(1) << 60) / channels, "p3d_sparse_validate: too many values");
    unsigned long long *first = reinterpret_cast<unsigned long long *>(first_bad);
    P3D_CUDA(ctx, cudaMemsetAsync(first, 0x7F, sizeof(int64_t), ctx->stream));  // 0x7F7F... = no error
    if (n == 0) return P3D_OK;
    if (coords) {
        // every coordinate inside the shape then packs into a 16-bit-per-field key
        if (batch > 65536 || sx > 32768 || sy > 32768 || sz > 32768)
            return set_error(ctx, P3D_ERR_UNSUPPORTED,
                             "p3d_sparse_validate: batch above 65536 or a spatial extent above 32768");
        P3D_REQUIRE(ctx, ws && (reinterpret_cast<uintptr_t>(ws) & 255) == 0 &&
                             ws_bytes >= p3d_sparse_validate_workspace(n),
                    "p3d_sparse_validate: workspace too small or not 256-byte aligned");
        P3D_REQUIRE(ctx, n < (int64_t(1) << 31), "p3d_sparse_validate: too many points");
        const int64_t cap = p3d_coord_hash_capacity(n);
        uint64_t *keys = static_cast<uint64_t *>(ws);
        int32_t *vals = reinterpret_cast<int32_t *>(keys + cap);
        fill_u64_kernel<<<blocks_for(cap, 256), 256, 0, ctx->stream>>>(keys, cap, kEmpty);
        int rc = check_launch(ctx, "fill_u64");
        if (rc) return rc;
        fill_i32_kernel<<<blocks_for(cap, 256), 256, 0, ctx->stream>>>(vals, cap, 0x7FFFFFFF);
        if ((rc = check_launch(ctx, "fill_i32"))) return rc;
        const int4 *c4 = reinterpret_cast<const int4 *>(coords);
        validate_insert_kernel<<<blocks_for(n, 256), 256, 0, ctx->stream>>>(c4, n, keys, vals,
                                                                            static_cast<uint64_t>(cap - 1), ctx->fault);
        if ((rc = check_launch(ctx, "validate_insert"))) return rc;
        validate_points_kernel<<<blocks_for(n, 256), 256, 0, ctx->stream>>>(
            c4, n, batch, sx, sy, sz, keys, vals, static_cast<uint64_t>(cap - 1), first);
        if ((rc = check_launch(ctx, "validate_points"))) return rc;
    }
    if (feats) {
        const int64_t count = n * channels;
        validate_finite_kernel<<<blocks_for(count, 256), 256, 0, ctx->stream>>>(feats, count, channels, first);
        return check_launch(ctx, "validate_finite");
    }
    return P3D_OK;
}

extern "C" int p3d_neighbor_map27_ws(p3d_ctx *ctx, const int32_t *coords, int64_t n, void *ws, size_t ws_bytes,
                                     int32_t *nbr_out) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, ws && (reinterpret_cast<uintptr_t>(ws) & 255) == 0, "p3d_neighbor_map27_ws: ws must be 256-byte aligned");
    P3D_REQUIRE(ctx, ws_bytes >= p3d_neighbor_map27_workspace(n), "p3d_neighbor_map27_ws: workspace too small");
    const int64_t cap = p3d_coord_hash_capacity(n);
    uint64_t *keys = static_cast<uint64_t *>(ws);
    int32_t *vals = reinterpret_cast<int32_t *>(keys + cap);
    int rc = p3d_coord_hash_build(ctx, coords, n, keys, vals, cap);
    if (rc) return rc;
    return p3d_neighbor_map27(ctx, coords, n, keys, vals, cap, nbr_out);
}

extern "C" int p3d_downsample_topology(p3d_ctx *ctx, const int32_t *coords, int64_t n, int batch, int sx, int sy,
                                       int sz, int factor, int32_t *grid, int32_t *out_coords, int32_t *parent,
                                       int32_t *child, int64_t *out_m) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, coords && grid && out_coords && parent && child && out_m, "p3d_downsample_topology: null pointer");
    P3D_REQUIRE(ctx, factor >= 1 && factor <= 4 && batch > 0 && sx > 0 && sy > 0 && sz > 0,
                "p3d_downsample_topology: bad shape or factor (1..4)");
    const int gx = (sx + factor - 1) / factor, gy = (sy + factor - 1) / factor, gz = (sz + factor - 1) / factor;
    const int64_t cells = static_cast<int64_t>(batch) * gx * gy * gz;
    P3D_REQUIRE(ctx, cells < (int64_t(1) << 30), "p3d_downsample_topology: grid too large");
    const int nchild = factor * factor * factor;
    // grid layout: [cells] flags->ranks, [ceil(cells/1024)+1] scan scratch, [1] total.
    int32_t *scratch = grid + cells;
    int32_t *total = scratch + ceil_div(cells, kScanBlock) + 1;
    P3D_CUDA(ctx, cudaMemsetAsync(grid, 0, sizeof(int32_t) * cells, ctx->stream));
    fill_i32_kernel<<<blocks_for(n * nchild, 256), 256, 0, ctx->stream>>>(child, n * nchild, -1);
    int rc = check_launch(ctx, "fill_i32");
    if (rc) return rc;
    if (n > 0) {
        down_mark_kernel<<<blocks_for(n, 256), 256, 0, ctx->stream>>>(reinterpret_cast<const int4 *>(coords), n, batch,
                                                                      sx, sy, sz, factor, gx, gy, gz, grid, ctx->fault);
        if ((rc = check_launch(ctx, "down_mark"))) return rc;
    }
    if ((rc = exclusive_scan(ctx, grid, cells, grid, scratch, total))) return rc;
    if (n > 0) {
        down_assign_kernel<<<blocks_for(n, 256), 256, 0, ctx->stream>>>(
            reinterpret_cast<const int4 *>(coords), n, batch, sx, sy, sz, factor, gx, gy, gz, grid, parent, child,
            reinterpret_cast<int4 *>(out_coords));
        if ((rc = check_launch(ctx, "down_assign"))) return rc;
    }
    i32_to_i64_kernel<<<1, 1, 0, ctx->stream>>>(total, out_m);
    return check_launch(ctx, "i32_to_i64");
}

extern "C" int64_t p3d_downsample_grid_ints(int batch, int sx, int sy, int sz, int factor) {
    const int64_t gx = (sx + factor - 1) / factor, gy = (sy + factor - 1) / factor, gz = (sz + factor - 1) / factor;
    const int64_t cells = static_cast<int64_t>(batch) * gx * gy * gz;
    return cells + ceil_div(cells, kScanBlock) + 2;
}

extern "C" int p3d_downsample_mean(p3d_ctx *ctx, const void *x, int64_t m, int channels, int factor,
                                   const int32_t *child, int dtype, void *out) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && child && out && channels > 0, "p3d_downsample_mean: bad argument");
    if (m == 0) return P3D_OK;
    const int nchild = factor * factor * factor;
    const unsigned grid = blocks_for(m, 8);
    if (dtype == P3D_F32 && nchild == 8 && channels % 4 == 0 &&
        ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
        down_mean8_f32_kernel<<<grid, 256, 0, ctx->stream>>>(static_cast<const float *>(x), m, channels, child,
                                                              static_cast<float *>(out));
        return check_launch(ctx, "down_mean");
    }
    P3D_DISPATCH(dtype, T,
                 down_mean_kernel<T><<<grid, 256, 0, ctx->stream>>>(static_cast<const T *>(x), m, channels, nchild,
                                                                    child, static_cast<T *>(out)));
    return check_launch(ctx, "down_mean");
}

extern "C" int p3d_upsample_nearest(p3d_ctx *ctx, const void *x, int64_t n, int channels, const int32_t *parent,
                                    int dtype, void *out) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && parent && out && channels > 0, "p3d_upsample_nearest: bad argument");
    if (n == 0) return P3D_OK;
    const unsigned grid = blocks_for(n, 8);
    if (dtype == P3D_F32)
        gather_rows_kernel<float><<<grid, 256, 0, ctx->stream>>>(static_cast<const float *>(x), n, channels, parent,
                                                                 static_cast<float *>(out));
    else  // bf16 and f16 rows are copied bit for bit
        gather_rows_kernel<uint16_t><<<grid, 256, 0, ctx->stream>>>(static_cast<const uint16_t *>(x), n, channels,
                                                                    parent, static_cast<uint16_t *>(out));
    return check_launch(ctx, "upsample_nearest");
}

extern "C" int p3d_c2s_topology(p3d_ctx *ctx, const int32_t *coords, int64_t n, int factor, const float *mask,
                                int64_t *scratch, int32_t *out_coords, int32_t *src_row, int8_t *src_child,
                                int64_t *out_m) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, coords && scratch && out_coords && src_row && src_child && out_m, "p3d_c2s_topology: null pointer");
    P3D_REQUIRE(ctx, factor >= 1 && factor <= 4, "p3d_c2s_topology: factor must be 1..4");
    P3D_REQUIRE(ctx, n * factor * factor * factor < (int64_t(1) << 31), "p3d_c2s_topology: too many points");
    // scratch (n+1 int64 = 2n+2 int32): [n] counts->offsets, [ceil(n/1024)+1] scan scratch, [1] total
    int32_t *counts = reinterpret_cast<int32_t *>(scratch);
    int32_t *sc = counts + n;
    int32_t *total = sc + ceil_div(n, kScanBlock) + 1;
    P3D_REQUIRE(ctx, n + ceil_div(n, kScanBlock) + 2 <= 2 * n + 2, "p3d_c2s_topology: scratch too small");
    const int nchild = factor * factor * factor;
    int rc;
    if (n > 0) {
        c2s_count_kernel<<<blocks_for(n, 256), 256, 0, ctx->stream>>>(n, nchild, mask, counts);
        if ((rc = check_launch(ctx, "c2s_count"))) return rc;
    }
    if ((rc = exclusive_scan(ctx, counts, n, counts, sc, total))) return rc;
    if (n > 0) {
        c2s_emit_kernel<<<blocks_for(n, 256), 256, 0, ctx->stream>>>(reinterpret_cast<const int4 *>(coords), n, factor,
                                                                     mask, counts, reinterpret_cast<int4 *>(out_coords),
                                                                     src_row, src_child);
        if ((rc = check_launch(ctx, "c2s_emit"))) return rc;
    }
    i32_to_i64_kernel<<<1, 1, 0, ctx->stream>>>(total, out_m);
    return check_launch(ctx, "i32_to_i64");
}

extern "C" int p3d_batch_offsets(p3d_ctx *ctx, const int32_t *coords, int64_t n, int batch, int32_t *offsets) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, coords && offsets && batch > 0 && n >= 0 && n < (int64_t(1) << 31),
                "p3d_batch_offsets: bad argument");
    P3D_REQUIRE(ctx, (reinterpret_cast<uintptr_t>(coords) & 15) == 0, "p3d_batch_offsets: coords must be 16-byte aligned");
    batch_offsets_kernel<<<blocks_for(batch + 1, 128), 128, 0, ctx->stream>>>(reinterpret_cast<const int4 *>(coords), n,
                                                                             batch, offsets);
    return check_launch(ctx, "batch_offsets");
}

extern "C" int p3d_c2s_gather(p3d_ctx *ctx, const void *x, int64_t in_channels, const int32_t *src_row,
                              const int8_t *src_child, int64_t m, int cout, int repeat, int dtype, void *out) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && src_row && src_child && out && cout > 0 && repeat > 0 && cout <= in_channels,
                "p3d_c2s_gather: bad argument");
    if (m == 0) return P3D_OK;
    const unsigned grid = blocks_for(m, 8);
    if (dtype == P3D_F32)
        c2s_gather_kernel<float><<<grid, 256, 0, ctx->stream>>>(static_cast<const float *>(x), in_channels, src_row,
                                                                src_child, m, cout, repeat, static_cast<float *>(out));
    else  // bf16 and f16 rows are copied bit for bit
        c2s_gather_kernel<uint16_t><<<grid, 256, 0, ctx->stream>>>(static_cast<const uint16_t *>(x), in_channels,
                                                                   src_row, src_child, m, cout, repeat,
                                                                   static_cast<uint16_t *>(out));
    return check_launch(ctx, "c2s_gather");
}
