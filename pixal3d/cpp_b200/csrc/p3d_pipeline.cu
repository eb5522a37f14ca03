// SLat cascade glue on the device (reference src/pipeline.cpp): latent
// (de)normalization around each SLat stage and the shape decoder's
// coordinate hand-off to the 1024 grid.
//
// Normalization (normalize_slat_f32 :333-357, run_slat_stage_f32 :418-431):
//   normalize   y = (x - mean[c]) / std[c]
//   denormalize y = x * std[c] + mean[c]
// in IEEE f32 with the reference's operation order (no contraction), so the
// results are the reference's to the bit; a non-finite result latches
// P3D_ERR_NONFINITE.  HBM-bound: one read and one write of [n][C] f32.
//
// Quantization (quantize_slat_coords_f32 :433-466, quantize_at_resolution
// :296-329): each coordinate axis maps to round((v + 0.5) / low * 63) in
// double precision (llround: halves away from zero) on the 64^3 grid of the
// 1024 cascade resolution; rows are then made unique in lexicographic
// (b, x, y, z) order.  Here that order comes from a per-batch 64^3
// occupancy grid: mark, count per 1024-cell block, scan the block counts,
// and emit each block's occupied cells at its offset (ranks inside a block
// from warp ballots) -- deterministic, no sort.
#include "p3d_common.cuh"

namespace p3d {
namespace {

constexpr int kGrid = 64;                               // 1024 / 16
constexpr int64_t kCells = int64_t(kGrid) * kGrid * kGrid;  // per batch item
constexpr int kScanBlock = 1024;                        // cells per block

__global__ void slat_norm_kernel(const float *__restrict__ x, int64_t total, int C, const float *__restrict__ mean,
                                 const float *__restrict__ stdv, int denorm, float *__restrict__ y, int *fault) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int c = static_cast<int>(i % C);
    const float v = denorm ? __fadd_rn(__fmul_rn(x[i], stdv[c]), mean[c]) : __fdiv_rn(__fsub_rn(x[i], mean[c]), stdv[c]);
    if (!isfinite(v)) latch_fault(fault, P3D_ERR_NONFINITE);
    y[i] = v;
}

__device__ __forceinline__ int quantize_axis(int v, int low) {
    const double mapped = (static_cast<double>(v) + 0.5) / static_cast<double>(low) * static_cast<double>(kGrid - 1);
    const long long r = llround(mapped);
    return (r < 0 || r >= kGrid) ? -1 : static_cast<int>(r);
}

__global__ void quantize_mark_kernel(const int4 *__restrict__ coords, int64_t n, int batch, int low,
                                     uint32_t *__restrict__ occ, int *fault) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int4 c = coords[i];
    const int qx = quantize_axis(c.y, low), qy = quantize_axis(c.z, low), qz = quantize_axis(c.w, low);
    if (c.x < 0 || c.x >= batch || qx < 0 || qy < 0 || qz < 0) {
        latch_fault(fault, P3D_ERR_INVALID);
        return;
    }
    occ[static_cast<int64_t>(c.x) * kCells + (static_cast<int64_t>(qx) * kGrid + qy) * kGrid + qz] = 1u;
}

__global__ void __launch_bounds__(kScanBlock) quantize_count_kernel(const uint32_t *__restrict__ occ,
                                                                    int32_t *__restrict__ block_count) {
    const int64_t cell = static_cast<int64_t>(blockIdx.x) * kScanBlock + threadIdx.x;
    const int cnt = __syncthreads_count(occ[cell] != 0u);
    if (threadIdx.x == 0) block_count[blockIdx.x] = cnt;
}

// Exclusive scan of block_count[0..m) into block_off[0..m], block_off[m] =
// total, by one block walking the array in chunks of 1024.
__global__ void __launch_bounds__(1024) quantize_scan_kernel(const int32_t *__restrict__ block_count, int64_t m,
                                                             int32_t *__restrict__ block_off, int64_t *count_out) {
    __shared__ int32_t warp_sum[32];
    __shared__ int32_t carry;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    if (t == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < m; base += 1024) {
        const int64_t i = base + t;
        const int32_t v = i < m ? block_count[i] : 0;
        int32_t s = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int32_t u = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += u;
        }
        if (lane == 31) warp_sum[warp] = s;
        __syncthreads();
        if (warp == 0) {
            int32_t w = warp_sum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int32_t u = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += u;
            }
            warp_sum[lane] = w;
        }
        __syncthreads();
        const int32_t incl = s + (warp > 0 ? warp_sum[warp - 1] : 0);
        if (i < m) block_off[i] = carry + incl - v;
        __syncthreads();
        if (t == 1023) carry += incl;
        __syncthreads();
    }
    if (t == 0) {
        block_off[m] = carry;
        *count_out = carry;
    }
}

__global__ void __launch_bounds__(kScanBlock) quantize_emit_kernel(const uint32_t *__restrict__ occ,
                                                                   const int32_t *__restrict__ block_off,
                                                                   int32_t *__restrict__ out) {
    __shared__ int32_t warp_cnt[kScanBlock / 32];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int64_t cell = static_cast<int64_t>(blockIdx.x) * kScanBlock + t;
    const bool on = occ[cell] != 0u;
    const unsigned ballot = __ballot_sync(0xffffffffu, on);
    if (lane == 0) warp_cnt[warp] = __popc(ballot);
    __syncthreads();
    if (!on) return;
    int rank = __popc(ballot & ((1u << lane) - 1u));
    for (int w = 0; w < warp; ++w) rank += warp_cnt[w];
    const int64_t pos = block_off[blockIdx.x] + rank;
    const int64_t b = cell / kCells, r = cell - b * kCells;
    reinterpret_cast<int4 *>(out)[pos] =
        make_int4(static_cast<int>(b), static_cast<int>(r / (kGrid * kGrid)), static_cast<int>((r / kGrid) % kGrid),
                  static_cast<int>(r % kGrid));
}

}  // namespace
}  // namespace p3d

using namespace p3d;

extern "C" int p3d_slat_normalize(p3d_ctx *ctx, const float *x, int64_t n, int channels, const float *mean,
                                  const float *stdv, int denormalize, float *out) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && mean && stdv && out && channels > 0 && n >= 0, "p3d_slat_normalize: bad argument");
    if (n == 0) return P3D_OK;
    DeviceGuard guard(ctx->device);
    const int64_t total = n * channels;
    slat_norm_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, ctx->stream>>>(
        x, total, channels, mean, stdv, denormalize ? 1 : 0, out, ctx->fault);
    return check_launch(ctx, "slat_normalize");
}

extern "C" size_t p3d_quantize_slat_coords_workspace(int batch) {
    if (batch <= 0) return 0;
    const int64_t cells = batch * kCells, blocks = cells / kScanBlock;
    return static_cast<size_t>(cells * 4 + (2 * blocks + 1) * 4 + 256);
}

extern "C" int p3d_quantize_slat_coords(p3d_ctx *ctx, const int32_t *coords, int64_t n, int batch, int low_resolution,
                                        int resolution, int32_t *out, int64_t *count, void *ws, size_t ws_bytes) {
    if (!ctx) return P3D_ERR_INVALID;
    if (resolution != 1024) return set_error(ctx, P3D_ERR_INVALID, "SLat cascade resolution must be 1024");
    if (low_resolution <= 0) return set_error(ctx, P3D_ERR_INVALID, "SLat cascade low resolution must be positive");
    P3D_REQUIRE(ctx, batch > 0 && batch <= 64 && n >= 0 && count && ws && (n == 0 || (coords && out)),
                "p3d_quantize_slat_coords: bad argument");
    P3D_REQUIRE(ctx, (reinterpret_cast<uintptr_t>(coords) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(ws) & 15) == 0,
                "p3d_quantize_slat_coords: coords, out and ws must be 16-byte aligned");
    P3D_REQUIRE(ctx, ws_bytes >= p3d_quantize_slat_coords_workspace(batch),
                "p3d_quantize_slat_coords: workspace too small");
    DeviceGuard guard(ctx->device);
    const int64_t cells = batch * kCells, blocks = cells / kScanBlock;
    uint32_t *occ = static_cast<uint32_t *>(ws);
    int32_t *bcount = reinterpret_cast<int32_t *>(occ + cells);
    int32_t *boff = bcount + blocks;
    P3D_CUDA(ctx, cudaMemsetAsync(occ, 0, sizeof(uint32_t) * cells, ctx->stream));
    if (n > 0) {
        quantize_mark_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(
            reinterpret_cast<const int4 *>(coords), n, batch, low_resolution, occ, ctx->fault);
        int rc = check_launch(ctx, "quantize_mark");
        if (rc) return rc;
    }
    quantize_count_kernel<<<static_cast<unsigned>(blocks), kScanBlock, 0, ctx->stream>>>(occ, bcount);
    int rc = check_launch(ctx, "quantize_count");
    if (rc) return rc;
    quantize_scan_kernel<<<1, 1024, 0, ctx->stream>>>(bcount, blocks, boff, count);
    if ((rc = check_launch(ctx, "quantize_scan"))) return rc;
    quantize_emit_kernel<<<static_cast<unsigned>(blocks), kScanBlock, 0, ctx->stream>>>(occ, boff, out);
    return check_launch(ctx, "quantize_emit");
}
