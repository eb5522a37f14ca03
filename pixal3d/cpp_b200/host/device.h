// Device staging for the host API: one p3d context per host thread, RAII
// device buffers, and uploads that convert host f32 to the kernels' 16-bit
// operand layout (zero-padded to the required row pitch).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

#include "p3d.h"
#include "pixal3d/sparse.h"

namespace pixal3d {
namespace b200 {

constexpr int kOperand = P3D_F16;  // 16-bit operand type of every contraction

// This thread's context on device $PIXAL3D_B200_DEVICE (default 0), legacy
// default stream.  Null (and *error set) when no sm_100 device is usable.
p3d_ctx *context(std::string *error);

// rc != P3D_OK -> false with the context's message in *error.
bool ok(p3d_ctx *ctx, int rc, std::string *error);
bool fail(std::string *error, const char *message);
bool fail(std::string *error, const std::string &message);

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

class Buffer {
public:
    Buffer() = default;
    ~Buffer() { reset(); }
    Buffer(const Buffer &) = delete;
    Buffer &operator=(const Buffer &) = delete;
    Buffer(Buffer &&o) noexcept { *this = std::move(o); }
    Buffer &operator=(Buffer &&o) noexcept {
        if (this != &o) {
            reset();
            ctx_ = o.ctx_;
            ptr_ = o.ptr_;
            bytes_ = o.bytes_;
            o.ptr_ = nullptr;
            o.bytes_ = 0;
        }
        return *this;
    }
    bool allocate(p3d_ctx *ctx, std::size_t bytes, std::string *error);
    void reset();
    template <typename T>
    T *as() const {
        return static_cast<T *>(ptr_);
    }
    void *get() const { return ptr_; }
    std::size_t bytes() const { return bytes_; }

private:
    p3d_ctx *ctx_ = nullptr;
    void *ptr_ = nullptr;
    std::size_t bytes_ = 0;
};

// Allocate `bytes` and copy host `src` into it.
bool upload(p3d_ctx *ctx, Buffer &dst, const void *src, std::size_t bytes, std::string *error);
bool download(p3d_ctx *ctx, void *dst, const Buffer &src, std::size_t bytes, std::string *error);

// Host f32 matrix [rows][cols] -> device 16-bit [rows][ld] (ld >= cols,
// extra columns zero).  src may be null when rows * cols == 0.
bool upload_operand(p3d_ctx *ctx, Buffer &dst, const float *src, int64_t rows, int64_t cols, int64_t ld,
                    std::string *error);

// Validity of a host sparse tensor, checked on the device: shape fields and
// sizes first, then p3d_sparse_validate on the uploaded coords / feats (the
// uploads are kept in *coords / *feats when given, to be reused).
bool validate_sparse(p3d_ctx *ctx, const SparseTensorF32 &t, Buffer *coords, Buffer *feats, std::string *error);
bool validate_varlen(p3d_ctx *ctx, const VarLenTensorF32 &t, Buffer *feats, std::string *error);

// Row offsets of each batch item (coords contiguous by batch, validated).
std::vector<int32_t> batch_offsets(const SparseTensorF32 &t);
std::vector<int32_t> varlen_offsets(const VarLenTensorF32 &t);

// Same batch/spatial shape and coords as `in`, `channels` feature columns.
void copy_shape(const SparseTensorF32 &in, int channels, SparseTensorF32 &out);

}  // namespace b200
}  // namespace pixal3d
