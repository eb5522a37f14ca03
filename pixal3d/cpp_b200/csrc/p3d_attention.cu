// Varlen flash attention over ragged voxel sequences (head_dim 64).
//
// Replaces sparse_scaled_dot_product_attention (src/sparse.cpp:704-783) and
// sparse_cross_attention (src/sparse.cpp:785-859): sequence s attends its
// query rows [cu_q[s], cu_q[s+1]) to key/value rows [cu_k[s], cu_k[s+1]).
// Online softmax (f32 running max / sum, exp2 with log2(e)-prescaled
// logits) replaces the reference's two-pass softmax; the N x N score matrix
// is never materialised (the reference GPU path materialises 512-query
// chunks, src/slat_flow.cpp:970-1000).
//
// CTA: 4 warps, 64 query rows (16 per warp) of one head; K/V streamed in
// 64-key tiles through double-buffered, XOR-swizzled shared memory
// (cp.async), fragments via ldmatrix, 16-bit mma.sync m16n8k16 with f32
// accumulation; P is re-packed from the S accumulators into A fragments
// without touching shared memory.
#include "p3d_common.cuh"

namespace p3d {
namespace {

constexpr int kD = 64;
constexpr int kBM = 64;
constexpr int kBN = 64;
constexpr int kThreadsAttn = 128;

__device__ __forceinline__ uint32_t swz(int row, int col) {
    // byte offset of element (row, col) in a [rows][64] bf16 tile, 16B chunks XOR row%8
    return static_cast<uint32_t>(row * 128 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
template <typename T>
__device__ __forceinline__ void mma16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                      uint32_t b1);
template <>
__device__ __forceinline__ void mma16<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                     uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16<__half>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Load `rows` x 64 bf16 rows (row r of the tile = global row base + r,
// valid while < limit) into a swizzled tile; 128 threads, 4 chunks each.
__device__ __forceinline__ void load_tile(uint8_t *tile, const uint16_t *base, int64_t ld, int64_t row0,
                                          int64_t limit) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int chunk = threadIdx.x + i * kThreadsAttn;  // 0..511
        const int r = chunk >> 3, c = chunk & 7;
        const int64_t gr = row0 + r;
        const bool ok = gr < limit;
        const uint16_t *src = base + (ok ? gr * ld : 0) + c * 8;
        cp_async16(tile + r * 128 + ((c ^ (r & 7)) << 4), src, ok ? 16u : 0u);
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreadsAttn)
    flash_attn_kernel(const uint16_t *__restrict__ q, int64_t ldq, const uint16_t *__restrict__ k,
                      int64_t ldk, const uint16_t *__restrict__ v, int64_t ldv, T *__restrict__ o,
                      int64_t ldo, const int32_t *__restrict__ cu_q, const int32_t *__restrict__ cu_k,
                      float scale_log2) {
    const int seq = blockIdx.z, head = blockIdx.y;
    const int64_t q0 = cu_q[seq], q1 = cu_q[seq + 1];
    const int64_t k0 = cu_k[seq], k1 = cu_k[seq + 1];
    const int64_t qt = q0 + static_cast<int64_t>(blockIdx.x) * kBM;
    if (qt >= q1 || k1 <= k0) return;

    __shared__ __align__(128) uint8_t sQ[kBM * 128];
    __shared__ __align__(128) uint8_t sK[2][kBN * 128];
    __shared__ __align__(128) uint8_t sV[2][kBN * 128];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint16_t *qh = q + head * kD;
    const uint16_t *kh = k + head * kD;
    const uint16_t *vh = v + head * kD;

    load_tile(sQ, qh, ldq, qt, q1);
    load_tile(sK[0], kh, ldk, k0, k1);
    load_tile(sV[0], vh, ldv, k0, k1);
    cp_async_commit();

    const int nblocks = static_cast<int>((k1 - k0 + kBN - 1) / kBN);
    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
    uint32_t qa[4][4];
    const uint32_t sq_base = smem_u32(sQ);

    for (int blk = 0; blk < nblocks; ++blk) {
        const int buf = blk & 1;
        if (blk + 1 < nblocks) {
            load_tile(sK[buf ^ 1], kh, ldk, k0 + (blk + 1) * kBN, k1);
            load_tile(sV[buf ^ 1], vh, ldv, k0 + (blk + 1) * kBN, k1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (blk == 0) {
            // Q fragments for this warp's 16 rows, 4 k-steps of 16.
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const int mi = lane >> 3, r = lane & 7;
                const int row = warp * 16 + (mi & 1) * 8 + r;
                const int col = kk * 16 + (mi >> 1) * 8;
                ldsm_x4(sq_base + swz(row, col), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
            }
        }
        const uint32_t sk_base = smem_u32(sK[buf]);
        const uint32_t sv_base = smem_u32(sV[buf]);
        // S = Q K^T : 16 x 64 per warp (8 n-tiles of 8 keys)
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {  // pairs of n-tiles
                const int mi = lane >> 3, r = lane & 7;
                const int key = jp * 16 + (mi >> 1) * 8 + r;
                const int col = kk * 16 + (mi & 1) * 8;
                uint32_t b0, b1, b2, b3;
                ldsm_x4(sk_base + swz(key, col), b0, b1, b2, b3);
                mma16<T>(s[2 * jp], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
                mma16<T>(s[2 * jp + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
            }
        }
        // mask keys past the end, scale into log2 domain, online softmax
        const int64_t kbase = k0 + static_cast<int64_t>(blk) * kBN;
        float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t kc = kbase + j * 8 + (lane & 3) * 2;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const bool valid = kc + (e & 1) < k1;
                s[j][e] = valid ? s[j][e] * scale_log2 : -INFINITY;
            }
            bm0 = fmaxf(bm0, fmaxf(s[j][0], s[j][1]));
            bm1 = fmaxf(bm1, fmaxf(s[j][2], s[j][3]));
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
            bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
            bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
        }
        const float nm0 = fmaxf(m0, bm0), nm1 = fmaxf(m1, bm1);
        const float a0 = exp2f(m0 - nm0), a1 = exp2f(m1 - nm1);
        m0 = nm0;
        m1 = nm1;
        float rs0 = 0.0f, rs1 = 0.0f;
        uint32_t pa[4][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float p0 = exp2f(s[j][0] - nm0), p1 = exp2f(s[j][1] - nm0);
            const float p2 = exp2f(s[j][2] - nm1), p3 = exp2f(s[j][3] - nm1);
            rs0 += p0 + p1;
            rs1 += p2 + p3;
            const int kk = j >> 1;
            if ((j & 1) == 0) {
                pa[kk][0] = pack2<T>(p0, p1);
                pa[kk][1] = pack2<T>(p2, p3);
            } else {
                pa[kk][2] = pack2<T>(p0, p1);
                pa[kk][3] = pack2<T>(p2, p3);
            }
        }
        l0 = l0 * a0 + rs0;
        l1 = l1 * a1 + rs1;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            acc[j][0] *= a0;
            acc[j][1] *= a0;
            acc[j][2] *= a1;
            acc[j][3] *= a1;
        }
        // O += P V : k = 64 keys (4 steps), n = 64 dims (8 tiles)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {
                const int mi = lane >> 3, r = lane & 7;
                const int key = kk * 16 + (mi & 1) * 8 + r;
                const int col = jp * 16 + (mi >> 1) * 8;
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(sv_base + swz(key, col), b0, b1, b2, b3);
                mma16<T>(acc[2 * jp], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
                mma16<T>(acc[2 * jp + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
            }
        }
        __syncthreads();
    }
    // row sums across the quad, normalise, store bf16
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
    const int64_t r0 = qt + warp * 16 + (lane >> 2);
    const int64_t r1 = r0 + 8;
    T *oh = o + head * kD;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int col = j * 8 + (lane & 3) * 2;
        if (r0 < q1) *reinterpret_cast<uint32_t *>(oh + r0 * ldo + col) = pack2<T>(acc[j][0] * inv0, acc[j][1] * inv0);
        if (r1 < q1) *reinterpret_cast<uint32_t *>(oh + r1 * ldo + col) = pack2<T>(acc[j][2] * inv1, acc[j][3] * inv1);
    }
}

}  // namespace
}  // namespace p3d

using namespace p3d;

extern "C" int p3d_varlen_attention(p3d_ctx *ctx, const void *q, int64_t ldq, const void *k, int64_t ldk,
                                    const void *v, int64_t ldv, void *out, int64_t ldo, const int32_t *cu_q,
                                    const int32_t *cu_k, int nseq, int64_t max_q, int heads, int head_dim,
                                    float scale, int dtype) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, q && k && v && out && cu_q && cu_k, "p3d_varlen_attention: null pointer");
    P3D_REQUIRE(ctx, head_dim == 64, "p3d_varlen_attention: head_dim must be 64");
    P3D_REQUIRE(ctx, is_16bit(dtype), "p3d_varlen_attention: dtype must be bf16 or f16");
    P3D_REQUIRE(ctx, heads > 0 && nseq > 0 && nseq < 65536, "p3d_varlen_attention: bad heads/nseq");
    P3D_REQUIRE(ctx, scale > 0.0f, "sparse attention scale must be finite and positive");
    P3D_REQUIRE(ctx, ldq % 8 == 0 && ldk % 8 == 0 && ldv % 8 == 0 && ldo % 2 == 0,
                "p3d_varlen_attention: leading dimensions must keep 16-byte rows");
    P3D_REQUIRE(ctx,
                ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) &
                 15) == 0,
                "p3d_varlen_attention: q/k/v must be 16-byte aligned");
    if (max_q <= 0) return P3D_OK;
    dim3 grid(static_cast<unsigned>(ceil_div(max_q, kBM)), heads, nseq);
    const float scale_log2 = scale * 1.4426950408889634f;
    const uint16_t *q16 = static_cast<const uint16_t *>(q), *k16 = static_cast<const uint16_t *>(k),
                   *v16 = static_cast<const uint16_t *>(v);
    if (dtype == P3D_BF16)
        flash_attn_kernel<__nv_bfloat16><<<grid, kThreadsAttn, 0, ctx->stream>>>(
            q16, ldq, k16, ldk, v16, ldv, static_cast<__nv_bfloat16 *>(out), ldo, cu_q, cu_k, scale_log2);
    else
        flash_attn_kernel<__half><<<grid, kThreadsAttn, 0, ctx->stream>>>(q16, ldq, k16, ldk, v16, ldv,
                                                                        static_cast<__half *>(out), ldo, cu_q, cu_k,
                                                                        scale_log2);
    return check_launch(ctx, "flash_attn");
}
