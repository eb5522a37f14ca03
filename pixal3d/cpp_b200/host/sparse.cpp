// Sparse-tensor operators of include/pixal3d/sparse.h on the B200 kernels.
// Each call: validate on the device, stage operands (16-bit, padded to the
// kernels' row pitch), run the kernel(s), copy the result back.
#include "pixal3d/sparse.h"

#include <cmath>

#include "device.h"
#include "ops_internal.h"

namespace pixal3d {

using b200::Buffer;
using b200::fail;
using b200::ok;

bool SparseTensorF32::valid(std::string *error) const {
    p3d_ctx *ctx = b200::context(error);
    return ctx && b200::validate_sparse(ctx, *this, nullptr, nullptr, error);
}

bool VarLenTensorF32::valid(std::string *error) const {
    p3d_ctx *ctx = b200::context(error);
    return ctx && b200::validate_varlen(ctx, *this, nullptr, error);
}

namespace b200 {

bool to_operand(p3d_ctx *ctx, const Buffer &dev_f32, const float *host, int64_t rows, int64_t cols, int64_t ld,
                Buffer &out, std::string *error) {
    if (ld != cols) return upload_operand(ctx, out, host, rows, cols, ld, error);
    const std::size_t count = static_cast<std::size_t>(rows * ld);
    if (!out.allocate(ctx, count * 2, error)) return false;
    return count == 0 ||
           ok(ctx, p3d_convert(ctx, dev_f32.get(), P3D_F32, static_cast<int64_t>(count), out.get(), kOperand), error);
}

bool linear_f32(p3d_ctx *ctx, const Buffer &x16, int64_t rows, int64_t kp, const float *w, const float *b, int cin,
                int cout, Buffer &y, std::string *error) {
    Buffer w16, bias;
    if (!upload_operand(ctx, w16, w, cout, cin, kp, error)) return false;
    if (b && !upload(ctx, bias, b, sizeof(float) * cout, error)) return false;
    if (!y.allocate(ctx, sizeof(float) * static_cast<std::size_t>(rows) * cout, error)) return false;
    if (rows == 0) return true;
    return ok(ctx,
              p3d_linear(ctx, x16.get(), kp, w16.get(), kOperand, b ? bias.as<float>() : nullptr, rows, cout, kp,
                         y.get(), cout, P3D_F32, P3D_EPI_NONE, nullptr, 0, nullptr, 0),
              error);
}

bool download_feats(p3d_ctx *ctx, const Buffer &y, std::size_t count, std::vector<float> &out, std::string *error) {
    out.resize(count);
    return download(ctx, out.data(), y, count * sizeof(float), error);
}

bool heads_to_64(p3d_ctx *ctx, const void *x16, int64_t ld, int64_t rows, int heads, int hd, Buffer &out,
                 std::string *error) {
    if (!out.allocate(ctx, static_cast<std::size_t>(rows) * heads * 64 * 2, error)) return false;
    return rows == 0 ||
           ok(ctx, p3d_repack_heads(ctx, x16, ld, rows, heads, hd, 64, out.get(), heads * 64, kOperand), error);
}

bool attention16(p3d_ctx *ctx, const void *q16, int64_t ldq, int64_t rows_q, const void *k16, int64_t ldk,
                 const void *v16, int64_t ldv, int64_t rows_k, const std::vector<int32_t> &cu_q,
                 const std::vector<int32_t> &cu_k, int heads, int hd, float scale, Buffer &out16, int64_t ld_out,
                 std::string *error) {
    if (hd > 64) return fail(error, "sparse attention head_dim above 64 is not supported by the B200 kernels");
    const int nseq = static_cast<int>(cu_q.size()) - 1;
    int64_t max_q = 0;
    for (int b = 0; b < nseq; ++b) max_q = std::max<int64_t>(max_q, cu_q[b + 1] - cu_q[b]);
    const int64_t w64 = static_cast<int64_t>(heads) * 64;
    Buffer q64, k64, v64, dcq, dck, o64;
    const void *qa = q16, *ka = k16, *va = v16;
    int64_t lq = ldq, lk = ldk, lv = ldv;
    if (hd != 64) {
        if (!heads_to_64(ctx, q16, ldq, rows_q, heads, hd, q64, error) ||
            !heads_to_64(ctx, k16, ldk, rows_k, heads, hd, k64, error) ||
            !heads_to_64(ctx, v16, ldv, rows_k, heads, hd, v64, error))
            return false;
        qa = q64.get(), ka = k64.get(), va = v64.get();
        lq = lk = lv = w64;
    }
    if (!upload(ctx, dcq, cu_q.data(), cu_q.size() * 4, error) || !upload(ctx, dck, cu_k.data(), cu_k.size() * 4, error))
        return false;
    const bool direct = hd == 64 && ld_out == w64;
    Buffer &o = direct ? out16 : o64;
    if (!o.allocate(ctx, static_cast<std::size_t>(rows_q) * w64 * 2, error)) return false;
    if (rows_q > 0 && max_q > 0 &&
        !ok(ctx,
            p3d_varlen_attention(ctx, qa, lq, ka, lk, va, lv, o.get(), w64, dcq.as<int32_t>(), dck.as<int32_t>(), nseq,
                                 max_q, rows_q, rows_k, heads, 64, scale, kOperand),
            error))
        return false;
    if (direct) return true;
    if (!out16.allocate(ctx, static_cast<std::size_t>(rows_q) * ld_out * 2, error)) return false;
    return rows_q == 0 ||
           ok(ctx, p3d_repack_heads(ctx, o64.get(), w64, rows_q, heads, 64, hd, out16.get(), ld_out, kOperand), error);
}

bool operand_to_host(p3d_ctx *ctx, const void *x16, int64_t rows, int64_t cols, int64_t ld, std::vector<float> &out,
                     std::string *error) {
    Buffer packed, y;
    const void *src = x16;
    if (ld != cols) {
        if (!packed.allocate(ctx, static_cast<std::size_t>(rows) * cols * 2, error)) return false;
        if (rows > 0 &&
            !ok(ctx, p3d_repack_heads(ctx, x16, ld, rows, 1, static_cast<int>(ld), static_cast<int>(cols),
                                      packed.get(), cols, kOperand),
                error))
            return false;
        src = packed.get();
    }
    if (!y.allocate(ctx, static_cast<std::size_t>(rows) * cols * 4, error)) return false;
    if (rows > 0 && !ok(ctx, p3d_convert(ctx, src, kOperand, rows * cols, y.get(), P3D_F32), error)) return false;
    return download_feats(ctx, y, static_cast<std::size_t>(rows) * cols, out, error);
}

}  // namespace b200

bool sparse_linear(const SparseTensorF32 &input, const float *weight, const float *bias, int out_channels,
                   SparseTensorF32 &output, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer x32;
    if (!b200::validate_sparse(ctx, input, nullptr, &x32, error)) return false;
    if (out_channels <= 0) return fail(error, "sparse output channel count must be positive");
    if (!weight) return fail(error, "sparse weight pointer is null");
    const int64_t n = static_cast<int64_t>(input.points());
    const int64_t kp = b200::round_up(input.channels, 8);
    Buffer x16, y;
    if (!b200::to_operand(ctx, x32, input.feats.data(), n, input.channels, kp, x16, error) ||
        !b200::linear_f32(ctx, x16, n, kp, weight, bias, input.channels, out_channels, y, error))
        return false;
    std::vector<float> feats;
    if (!b200::download_feats(ctx, y, static_cast<std::size_t>(n) * out_channels, feats, error)) return false;
    b200::copy_shape(input, out_channels, output);
    output.feats = std::move(feats);
    return true;
}

bool varlen_linear(const VarLenTensorF32 &input, const float *weight, const float *bias, int out_channels,
                   VarLenTensorF32 &output, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer x32;
    if (!b200::validate_varlen(ctx, input, &x32, error)) return false;
    if (out_channels <= 0) return fail(error, "sparse output channel count must be positive");
    if (!weight) return fail(error, "sparse weight pointer is null");
    const int64_t n = static_cast<int64_t>(input.offsets.back());
    const int64_t kp = b200::round_up(input.channels, 8);
    Buffer x16, y;
    if (!b200::to_operand(ctx, x32, input.feats.data(), n, input.channels, kp, x16, error) ||
        !b200::linear_f32(ctx, x16, n, kp, weight, bias, input.channels, out_channels, y, error))
        return false;
    std::vector<float> feats;
    if (!b200::download_feats(ctx, y, static_cast<std::size_t>(n) * out_channels, feats, error)) return false;
    output.batch_size = input.batch_size;
    output.channels = out_channels;
    output.offsets = input.offsets;
    output.feats = std::move(feats);
    return true;
}

bool sparse_layer_norm(const SparseTensorF32 &input, float epsilon, const float *gamma, const float *beta,
                       SparseTensorF32 &output, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer x32;
    if (!b200::validate_sparse(ctx, input, nullptr, &x32, error)) return false;
    if (!(epsilon > 0.0f) || !std::isfinite(epsilon))
        return fail(error, "sparse layer norm epsilon must be finite and positive");
    if ((gamma == nullptr) != (beta == nullptr))
        return fail(error, "sparse layer norm affine parameters must be both null or non-null");
    const int64_t n = static_cast<int64_t>(input.points());
    const int c = input.channels;
    Buffer g, b, y;
    if (gamma && (!b200::upload(ctx, g, gamma, sizeof(float) * c, error) ||
                  !b200::upload(ctx, b, beta, sizeof(float) * c, error)))
        return false;
    if (!y.allocate(ctx, sizeof(float) * static_cast<std::size_t>(n) * c, error)) return false;
    if (n > 0 && !ok(ctx,
                     p3d_layernorm_modulate(ctx, x32.as<float>(), n, c, epsilon, gamma ? g.as<float>() : nullptr,
                                            gamma ? b.as<float>() : nullptr, nullptr, 0, nullptr, 0, y.get(), P3D_F32),
                     error))
        return false;
    std::vector<float> feats;
    if (!b200::download_feats(ctx, y, static_cast<std::size_t>(n) * c, feats, error)) return false;
    b200::copy_shape(input, c, output);
    output.feats = std::move(feats);
    return true;
}

bool sparse_downsample_mean(const SparseTensorF32 &input, int factor, SparseTensorF32 &output, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer c32, x32;
    if (!b200::validate_sparse(ctx, input, &c32, &x32, error)) return false;
    if (factor <= 0) return fail(error, "sparse downsample factor must be positive");
    if (factor > 4) return fail(error, "sparse downsample factor above 4 is not supported by the B200 kernels");
    const int64_t n = static_cast<int64_t>(input.points());
    const int c = input.channels;
    const int nchild = factor * factor * factor;
    const int64_t gints = p3d_downsample_grid_ints(input.batch_size, input.spatial_x, input.spatial_y,
                                                   input.spatial_z, factor);
    Buffer grid, oc, parent, child, dm, y;
    if (!grid.allocate(ctx, sizeof(int32_t) * gints, error) || !oc.allocate(ctx, sizeof(int32_t) * 4 * n, error) ||
        !parent.allocate(ctx, sizeof(int32_t) * n, error) || !child.allocate(ctx, sizeof(int32_t) * n * nchild, error) ||
        !dm.allocate(ctx, 8, error))
        return false;
    if (!ok(ctx,
            p3d_downsample_topology(ctx, c32.as<int32_t>(), n, input.batch_size, input.spatial_x, input.spatial_y,
                                    input.spatial_z, factor, grid.as<int32_t>(), oc.as<int32_t>(),
                                    parent.as<int32_t>(), child.as<int32_t>(), dm.as<int64_t>()),
            error))
        return false;
    int64_t m = 0;
    if (!b200::download(ctx, &m, dm, 8, error)) return false;
    if (!y.allocate(ctx, sizeof(float) * static_cast<std::size_t>(m) * c, error)) return false;
    if (m > 0 && !ok(ctx, p3d_downsample_mean(ctx, x32.get(), m, c, factor, child.as<int32_t>(), P3D_F32, y.get()),
                     error))
        return false;
    std::vector<int32_t> coords(static_cast<std::size_t>(m) * 4);
    std::vector<float> feats;
    if (!b200::download(ctx, coords.data(), oc, coords.size() * 4, error) ||
        !b200::download_feats(ctx, y, static_cast<std::size_t>(m) * c, feats, error))
        return false;
    output.batch_size = input.batch_size;
    output.channels = c;
    output.spatial_x = (input.spatial_x + factor - 1) / factor;
    output.spatial_y = (input.spatial_y + factor - 1) / factor;
    output.spatial_z = (input.spatial_z + factor - 1) / factor;
    output.coords = std::move(coords);
    output.feats = std::move(feats);
    return true;
}

bool sparse_channel_to_spatial(const SparseTensorF32 &input, int factor, const SparseTensorF32 *subdivision,
                               SparseTensorF32 &output, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer c32, x32, m32;
    if (!b200::validate_sparse(ctx, input, &c32, &x32, error)) return false;
    if (factor <= 0) return fail(error, "sparse channel-to-spatial factor must be positive");
    const int nchild = factor * factor * factor;
    if (input.channels % nchild != 0)
        return fail(error, "sparse channel-to-spatial channels are not divisible by factor^3");
    if (subdivision) {
        if (!b200::validate_sparse(ctx, *subdivision, nullptr, &m32, error) ||
            subdivision->batch_size != input.batch_size || subdivision->channels != nchild ||
            subdivision->coords != input.coords)
            return fail(error, "sparse subdivision shape or coordinates do not match input");
    }
    const int64_t n = static_cast<int64_t>(input.points());
    const int cout = input.channels / nchild;
    Buffer scratch, oc, src_row, src_child, dm, y;
    if (!scratch.allocate(ctx, sizeof(int64_t) * (n + 1), error) ||
        !oc.allocate(ctx, sizeof(int32_t) * 4 * n * nchild, error) ||
        !src_row.allocate(ctx, sizeof(int32_t) * n * nchild, error) || !src_child.allocate(ctx, n * nchild, error) ||
        !dm.allocate(ctx, 8, error))
        return false;
    if (!ok(ctx,
            p3d_c2s_topology(ctx, c32.as<int32_t>(), n, factor, subdivision ? m32.as<float>() : nullptr,
                             scratch.as<int64_t>(), oc.as<int32_t>(), src_row.as<int32_t>(), src_child.as<int8_t>(),
                             dm.as<int64_t>()),
            error))
        return false;
    int64_t m = 0;
    if (!b200::download(ctx, &m, dm, 8, error)) return false;
    if (!y.allocate(ctx, sizeof(float) * static_cast<std::size_t>(m) * cout, error)) return false;
    if (m > 0 && !ok(ctx,
                     p3d_c2s_gather(ctx, x32.get(), input.channels, src_row.as<int32_t>(), src_child.as<int8_t>(), m,
                                    cout, 1, P3D_F32, y.get()),
                     error))
        return false;
    std::vector<int32_t> coords(static_cast<std::size_t>(m) * 4);
    std::vector<float> feats;
    if (!b200::download(ctx, coords.data(), oc, coords.size() * 4, error) ||
        !b200::download_feats(ctx, y, static_cast<std::size_t>(m) * cout, feats, error))
        return false;
    output.batch_size = input.batch_size;
    output.channels = cout;
    output.spatial_x = input.spatial_x * factor;
    output.spatial_y = input.spatial_y * factor;
    output.spatial_z = input.spatial_z * factor;
    output.coords = std::move(coords);
    output.feats = std::move(feats);
    return true;
}

bool sparse_scaled_dot_product_attention(const SparseTensorF32 &query, const SparseTensorF32 &key,
                                         const SparseTensorF32 &value, int num_heads, int head_dim, float scale,
                                         SparseTensorF32 &output, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer q32, k32, v32;
    if (!b200::validate_sparse(ctx, query, nullptr, &q32, error) ||
        !b200::validate_sparse(ctx, key, nullptr, &k32, error) ||
        !b200::validate_sparse(ctx, value, nullptr, &v32, error))
        return false;
    if (num_heads <= 0 || head_dim <= 0 || query.channels != num_heads * head_dim ||
        key.channels != query.channels || value.channels != query.channels)
        return fail(error, "sparse attention channel/head dimensions are invalid");
    if (query.batch_size != key.batch_size || query.batch_size != value.batch_size)
        return fail(error, "sparse attention batch sizes do not match");
    if (!(scale > 0.0f) || !std::isfinite(scale))
        return fail(error, "sparse attention scale must be finite and positive");
    const std::vector<int32_t> cq = b200::batch_offsets(query), ck = b200::batch_offsets(key),
                               cv = b200::batch_offsets(value);
    for (int b = 0; b < query.batch_size; ++b)
        if ((cq[b + 1] > cq[b] && ck[b + 1] == ck[b]) || ck[b + 1] - ck[b] != cv[b + 1] - cv[b])
            return fail(error, "sparse attention has no keys or mismatched key/value rows");
    const int c = query.channels;
    const int64_t ld = b200::round_up(c, 8);
    const int64_t nq = static_cast<int64_t>(query.points()), nk = static_cast<int64_t>(key.points());
    Buffer q16, k16, v16, o;
    if (!b200::to_operand(ctx, q32, query.feats.data(), nq, c, ld, q16, error) ||
        !b200::to_operand(ctx, k32, key.feats.data(), nk, c, ld, k16, error) ||
        !b200::to_operand(ctx, v32, value.feats.data(), nk, c, ld, v16, error) ||
        !b200::attention16(ctx, q16.get(), ld, nq, k16.get(), ld, v16.get(), ld, nk, cq, ck, num_heads, head_dim,
                           scale, o, c, error))
        return false;
    std::vector<float> feats;
    if (!b200::operand_to_host(ctx, o.get(), nq, c, c, feats, error)) return false;
    b200::copy_shape(query, c, output);
    output.feats = std::move(feats);
    return true;
}

bool sparse_cross_attention(const SparseTensorF32 &query, const VarLenTensorF32 &key, const VarLenTensorF32 &value,
                            int num_heads, int head_dim, float scale, SparseTensorF32 &output, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer q32, k32, v32;
    if (!b200::validate_sparse(ctx, query, nullptr, &q32, error) || !b200::validate_varlen(ctx, key, &k32, error) ||
        !b200::validate_varlen(ctx, value, &v32, error))
        return false;
    if (key.batch_size != value.batch_size || key.offsets != value.offsets || key.batch_size != query.batch_size ||
        num_heads <= 0 || head_dim <= 0 || query.channels != num_heads * head_dim ||
        key.channels != query.channels || value.channels != query.channels)
        return fail(error, "sparse cross-attention dimensions or offsets are invalid");
    if (!(scale > 0.0f) || !std::isfinite(scale))
        return fail(error, "sparse attention scale must be finite and positive");
    const std::vector<int32_t> cq = b200::batch_offsets(query), ck = b200::varlen_offsets(key);
    for (int b = 0; b < query.batch_size; ++b)
        if (cq[b + 1] > cq[b] && ck[b + 1] == ck[b])
            return fail(error, "sparse cross-attention has an empty key sequence");
    const int c = query.channels;
    const int64_t ld = b200::round_up(c, 8);
    const int64_t nq = static_cast<int64_t>(query.points()), nk = static_cast<int64_t>(key.offsets.back());
    Buffer q16, k16, v16, o;
    if (!b200::to_operand(ctx, q32, query.feats.data(), nq, c, ld, q16, error) ||
        !b200::to_operand(ctx, k32, key.feats.data(), nk, c, ld, k16, error) ||
        !b200::to_operand(ctx, v32, value.feats.data(), nk, c, ld, v16, error) ||
        !b200::attention16(ctx, q16.get(), ld, nq, k16.get(), ld, v16.get(), ld, nk, cq, ck, num_heads, head_dim,
                           scale, o, c, error))
        return false;
    std::vector<float> feats;
    if (!b200::operand_to_host(ctx, o.get(), nq, c, c, feats, error)) return false;
    b200::copy_shape(query, c, output);
    output.feats = std::move(feats);
    return true;
}

namespace {
// RoPE and/or per-head RMS norm of n rows in place on the 16-bit operand.
bool heads_norm_rope(p3d_ctx *ctx, const Buffer &x32, const float *host, int64_t n, int c, int heads, int hd,
                     const float *gamma, const Buffer *coords, float fmin, float fbase, std::vector<float> &out,
                     std::string *error) {
    const int64_t ld = b200::round_up(c, 8);
    Buffer x16, g;
    if (!b200::to_operand(ctx, x32, host, n, c, ld, x16, error)) return false;
    if (gamma && !b200::upload(ctx, g, gamma, sizeof(float) * c, error)) return false;
    if (n > 0 && !ok(ctx,
                     p3d_qk_rmsnorm_rope(ctx, x16.get(), n, ld, heads, hd, gamma ? g.as<float>() : nullptr,
                                         coords ? coords->as<int32_t>() : nullptr, fmin, fbase, b200::kOperand),
                     error))
        return false;
    return b200::operand_to_host(ctx, x16.get(), n, c, ld, out, error);
}

bool heads_ok(int c, int heads, int hd) { return heads > 0 && hd > 0 && hd % 2 == 0 && hd <= 64 && c == heads * hd; }
}  // namespace

bool sparse_rotary_position_embedding(const SparseTensorF32 &input, int num_heads, int head_dim, float frequency_min,
                                      float frequency_base, SparseTensorF32 &output, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer c32, x32;
    if (!b200::validate_sparse(ctx, input, &c32, &x32, error)) return false;
    if (!heads_ok(input.channels, num_heads, head_dim)) return fail(error, "sparse RoPE head dimensions are invalid");
    if (!(frequency_min > 0.0f) || !(frequency_base > 0.0f) || !std::isfinite(frequency_min) ||
        !std::isfinite(frequency_base))
        return fail(error, "sparse RoPE frequencies must be finite and positive");
    std::vector<float> feats;
    if (!heads_norm_rope(ctx, x32, input.feats.data(), static_cast<int64_t>(input.points()), input.channels, num_heads,
                         head_dim, nullptr, &c32, frequency_min, frequency_base, feats, error))
        return false;
    b200::copy_shape(input, input.channels, output);
    output.feats = std::move(feats);
    return true;
}

bool sparse_multihead_rms_norm(const SparseTensorF32 &input, int num_heads, int head_dim, const float *gamma,
                               SparseTensorF32 &output, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer x32;
    if (!b200::validate_sparse(ctx, input, nullptr, &x32, error)) return false;
    if (!heads_ok(input.channels, num_heads, head_dim) || !gamma)
        return fail(error, "sparse multi-head RMS norm dimensions are invalid");
    std::vector<float> feats;
    if (!heads_norm_rope(ctx, x32, input.feats.data(), static_cast<int64_t>(input.points()), input.channels, num_heads,
                         head_dim, gamma, nullptr, 1.0f, 10000.0f, feats, error))
        return false;
    b200::copy_shape(input, input.channels, output);
    output.feats = std::move(feats);
    return true;
}

bool varlen_multihead_rms_norm(const VarLenTensorF32 &input, int num_heads, int head_dim, const float *gamma,
                               VarLenTensorF32 &output, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer x32;
    if (!b200::validate_varlen(ctx, input, &x32, error)) return false;
    if (!heads_ok(input.channels, num_heads, head_dim) || !gamma)
        return fail(error, "sparse multi-head RMS norm dimensions are invalid");
    std::vector<float> feats;
    if (!heads_norm_rope(ctx, x32, input.feats.data(), static_cast<int64_t>(input.offsets.back()), input.channels,
                         num_heads, head_dim, gamma, nullptr, 1.0f, 10000.0f, feats, error))
        return false;
    output.batch_size = input.batch_size;
    output.channels = input.channels;
    output.offsets = input.offsets;
    output.feats = std::move(feats);
    return true;
}

bool sparse_submanifold_conv3d(const SparseTensorF32 &input, const float *weight, const float *bias, int out_channels,
                               SparseTensorF32 &output, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer c32, x32;
    if (!b200::validate_sparse(ctx, input, &c32, &x32, error)) return false;
    if (out_channels <= 0) return fail(error, "sparse output channel count must be positive");
    if (!weight) return fail(error, "sparse weight pointer is null");
    const int64_t n = static_cast<int64_t>(input.points());
    const int cin = input.channels;
    const int64_t kp = b200::round_up(cin, 64);
    Buffer x16, w16, bb, ws, nbr, y;
    if (!b200::to_operand(ctx, x32, input.feats.data(), n, cin, kp, x16, error) ||
        !b200::upload_operand(ctx, w16, weight, 27LL * out_channels, cin, kp, error))
        return false;
    if (bias && !b200::upload(ctx, bb, bias, sizeof(float) * out_channels, error)) return false;
    const std::size_t wsb = p3d_neighbor_map27_workspace(n);
    if (!ws.allocate(ctx, wsb, error) || !nbr.allocate(ctx, sizeof(int32_t) * 27 * n, error) ||
        !y.allocate(ctx, sizeof(float) * static_cast<std::size_t>(n) * out_channels, error))
        return false;
    if (n > 0 &&
        (!ok(ctx, p3d_neighbor_map27_ws(ctx, c32.as<int32_t>(), n, ws.get(), wsb, nbr.as<int32_t>()), error) ||
         !ok(ctx,
             p3d_subm_conv3d(ctx, x16.get(), n, kp, nbr.as<int32_t>(), w16.get(), b200::kOperand,
                             bias ? bb.as<float>() : nullptr, out_channels, y.get(), out_channels, P3D_F32,
                             P3D_EPI_NONE, nullptr, 0, nullptr, 0),
             error)))
        return false;
    std::vector<float> feats;
    if (!b200::download_feats(ctx, y, static_cast<std::size_t>(n) * out_channels, feats, error)) return false;
    b200::copy_shape(input, out_channels, output);
    output.feats = std::move(feats);
    return true;
}

}  // namespace pixal3d
