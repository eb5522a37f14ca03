// C ABI entry of the varlen attention (the tcgen05 kernel is in p3d_fmha.cu).
//
// Replaces sparse_scaled_dot_product_attention (src/sparse.cpp:704-783),
// sparse_cross_attention (src/sparse.cpp:785-859) and the query-chunked ggml
// attention of the reference GPU path (src/slat_flow.cpp:947-1001).
#include "p3d_common.cuh"

int p3d_fmha_tc(p3d_ctx *ctx, const void *q, int64_t ldq, const void *k, int64_t ldk, const void *v, int64_t ldv,
                void *out, int64_t ldo, const int32_t *cu_q, const int32_t *cu_k, int nseq, int64_t max_q,
                int64_t rows_q, int64_t rows_k, int heads, float scale, int dtype);

using namespace p3d;

extern "C" int p3d_varlen_attention(p3d_ctx *ctx, const void *q, int64_t ldq, const void *k, int64_t ldk,
                                    const void *v, int64_t ldv, void *out, int64_t ldo, const int32_t *cu_q,
                                    const int32_t *cu_k, int nseq, int64_t max_q, int64_t rows_q, int64_t rows_k,
                                    int heads, int head_dim, float scale, int dtype) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, q && k && v && out && cu_q && cu_k, "p3d_varlen_attention: null pointer");
    P3D_REQUIRE(ctx, head_dim == 64, "p3d_varlen_attention: head_dim must be 64");
    P3D_REQUIRE(ctx, is_16bit(dtype), "p3d_varlen_attention: dtype must be bf16 or f16");
    P3D_REQUIRE(ctx, heads > 0 && heads < 65536 && nseq > 0 && nseq < 65536, "p3d_varlen_attention: bad heads/nseq");
    P3D_REQUIRE(ctx, scale > 0.0f, "sparse attention scale must be finite and positive");
    P3D_REQUIRE(ctx, ldq % 8 == 0 && ldk % 8 == 0 && ldv % 8 == 0 && ldo % 8 == 0,
                "p3d_varlen_attention: leading dimensions must keep 16-byte rows");
    P3D_REQUIRE(ctx,
                ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
                  reinterpret_cast<uintptr_t>(out)) & 15) == 0,
                "p3d_varlen_attention: q/k/v/out must be 16-byte aligned");
    P3D_REQUIRE(ctx, rows_q >= 0 && rows_k > 0 && rows_q < (int64_t(1) << 31) && rows_k < (int64_t(1) << 31),
                "p3d_varlen_attention: bad row counts");
    if (max_q <= 0 || rows_q == 0) return P3D_OK;
    return p3d_fmha_tc(ctx, q, ldq, k, ldk, v, ldv, out, ldo, cu_q, cu_k, nseq, max_q, rows_q, rows_k, heads, scale,
                       dtype);
}
