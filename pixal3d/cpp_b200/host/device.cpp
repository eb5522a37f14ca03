#include "device.h"

#include <cmath>
#include <cstdlib>
#include <memory>

namespace pixal3d {
namespace b200 {

namespace {
struct CtxHolder {
    p3d_ctx *ctx = nullptr;
    int rc = P3D_OK;
    ~CtxHolder() {
        if (ctx) p3d_ctx_destroy(ctx);
    }
};
}  // namespace

p3d_ctx *context(std::string *error) {
    thread_local CtxHolder holder;
    thread_local bool tried = false;
    if (!tried) {
        tried = true;
        const char *env = std::getenv("PIXAL3D_B200_DEVICE");
        const int device = env ? std::atoi(env) : 0;
        holder.rc = p3d_ctx_create(device, nullptr, &holder.ctx);
    }
    if (!holder.ctx && error) *error = "no usable B200 (sm_100) device for the pixal3d B200 path";
    return holder.ctx;
}

bool fail(std::string *error, const char *message) {
    if (error) *error = message;
    return false;
}

bool fail(std::string *error, const std::string &message) {
    if (error) *error = message;
    return false;
}

bool ok(p3d_ctx *ctx, int rc, std::string *error) {
    if (rc == P3D_OK) return true;
    if (error) *error = ctx ? p3d_last_error(ctx) : "p3d call failed";
    if (error && error->empty()) *error = "p3d status " + std::to_string(rc);
    return false;
}

bool Buffer::allocate(p3d_ctx *ctx, std::size_t bytes, std::string *error) {
    reset();
    ctx_ = ctx;
    if (!ok(ctx, p3d_device_alloc(ctx, bytes, &ptr_), error)) return false;
    bytes_ = bytes;
    return true;
}

void Buffer::reset() {
    if (ptr_ && ctx_) p3d_device_free(ctx_, ptr_);
    ptr_ = nullptr;
    bytes_ = 0;
}

bool upload(p3d_ctx *ctx, Buffer &dst, const void *src, std::size_t bytes, std::string *error) {
    if (!dst.allocate(ctx, bytes, error)) return false;
    return bytes == 0 || ok(ctx, p3d_copy_to_device(ctx, dst.get(), src, bytes), error);
}

bool download(p3d_ctx *ctx, void *dst, const Buffer &src, std::size_t bytes, std::string *error) {
    if (bytes == 0) return true;
    return ok(ctx, p3d_copy_to_host(ctx, dst, src.get(), bytes), error) && ok(ctx, p3d_ctx_check(ctx), error);
}

bool upload_operand(p3d_ctx *ctx, Buffer &dst, const float *src, int64_t rows, int64_t cols, int64_t ld,
                    std::string *error) {
    const std::size_t count = static_cast<std::size_t>(rows) * static_cast<std::size_t>(ld);
    Buffer staged;
    if (ld == cols || rows == 0) {
        if (!upload(ctx, staged, src, count * sizeof(float), error)) return false;
    } else {
        std::vector<float> padded(count, 0.0f);
        for (int64_t r = 0; r < rows; ++r)
            for (int64_t c = 0; c < cols; ++c) padded[r * ld + c] = src[r * cols + c];
        if (!upload(ctx, staged, padded.data(), count * sizeof(float), error)) return false;
    }
    if (!dst.allocate(ctx, count * 2, error)) return false;
    return ok(ctx, p3d_convert(ctx, staged.get(), P3D_F32, static_cast<int64_t>(count), dst.get(), kOperand), error);
}

namespace {
const char *kValidMessages[4] = {"sparse coordinate is outside its shape",
                                 "sparse coordinates contain a duplicate point",
                                 "sparse coordinates must be contiguous by batch",
                                 "sparse features contain a non-finite value"};
}  // namespace

bool validate_sparse(p3d_ctx *ctx, const SparseTensorF32 &t, Buffer *coords, Buffer *feats, std::string *error) {
    if (t.batch_size <= 0 || t.channels <= 0 || t.spatial_x <= 0 || t.spatial_y <= 0 || t.spatial_z <= 0)
        return fail(error, "invalid sparse tensor shape");
    if (t.coords.size() % 4 != 0) return fail(error, "sparse coordinates must have four columns");
    if (t.feats.size() != t.points() * static_cast<std::size_t>(t.channels))
        return fail(error, "sparse feature count does not match coordinates");
    Buffer lc, lf;
    Buffer &c = coords ? *coords : lc;
    Buffer &f = feats ? *feats : lf;
    const int64_t n = static_cast<int64_t>(t.points());
    if (!upload(ctx, c, t.coords.data(), t.coords.size() * sizeof(int32_t), error)) return false;
    if (!upload(ctx, f, t.feats.data(), t.feats.size() * sizeof(float), error)) return false;
    Buffer ws, first;
    if (!ws.allocate(ctx, p3d_sparse_validate_workspace(n), error) || !first.allocate(ctx, 8, error)) return false;
    if (!ok(ctx,
            p3d_sparse_validate(ctx, c.as<int32_t>(), n, f.as<float>(), t.channels, t.batch_size, t.spatial_x,
                                t.spatial_y, t.spatial_z, ws.get(), ws.bytes(), first.as<int64_t>()),
            error))
        return false;
    int64_t r = 0;
    if (!download(ctx, &r, first, 8, error)) return false;
    if (r >= 0x7F7F7F7F7F7F7F7Fll) return true;
    return fail(error, kValidMessages[r & 3]);
}

bool validate_varlen(p3d_ctx *ctx, const VarLenTensorF32 &t, Buffer *feats, std::string *error) {
    if (t.batch_size <= 0 || t.channels <= 0 || t.offsets.size() != static_cast<std::size_t>(t.batch_size + 1) ||
        t.offsets.front() != 0)
        return fail(error, "invalid variable-length tensor shape");
    for (std::size_t i = 1; i < t.offsets.size(); ++i)
        if (t.offsets[i] < t.offsets[i - 1]) return fail(error, "variable-length tensor offsets are not monotonic");
    if (t.offsets.back() * static_cast<std::size_t>(t.channels) != t.feats.size())
        return fail(error, "variable-length tensor feature count does not match offsets");
    Buffer lf;
    Buffer &f = feats ? *feats : lf;
    if (!upload(ctx, f, t.feats.data(), t.feats.size() * sizeof(float), error)) return false;
    Buffer first;
    if (!first.allocate(ctx, 8, error)) return false;
    if (!ok(ctx,
            p3d_sparse_validate(ctx, nullptr, static_cast<int64_t>(t.offsets.back()), f.as<float>(), t.channels, 1, 1,
                                1, 1, nullptr, 0, first.as<int64_t>()),
            error))
        return false;
    int64_t r = 0;
    if (!download(ctx, &r, first, 8, error)) return false;
    if (r >= 0x7F7F7F7F7F7F7F7Fll) return true;
    return fail(error, "variable-length tensor contains a non-finite value");
}

std::vector<int32_t> batch_offsets(const SparseTensorF32 &t) {
    std::vector<int32_t> off(static_cast<std::size_t>(t.batch_size) + 1, 0);
    for (std::size_t p = 0; p < t.points(); ++p) off[static_cast<std::size_t>(t.coords[p * 4]) + 1]++;
    for (int b = 0; b < t.batch_size; ++b) off[b + 1] += off[b];
    return off;
}

std::vector<int32_t> varlen_offsets(const VarLenTensorF32 &t) {
    return std::vector<int32_t>(t.offsets.begin(), t.offsets.end());
}

void copy_shape(const SparseTensorF32 &in, int channels, SparseTensorF32 &out) {
    out.batch_size = in.batch_size;
    out.channels = channels;
    out.spatial_x = in.spatial_x;
    out.spatial_y = in.spatial_y;
    out.spatial_z = in.spatial_z;
    out.coords = in.coords;
}

}  // namespace b200
}  // namespace pixal3d
