// Building blocks shared by the host-API translation units.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "device.h"
#include "pixal3d/sparse_transformer.h"

namespace pixal3d {
namespace b200 {

// Device f32 -> 16-bit operand with row pitch ld (host copy used when ld > cols).
bool to_operand(p3d_ctx *ctx, const Buffer &dev_f32, const float *host, int64_t rows, int64_t cols, int64_t ld,
                Buffer &out, std::string *error);
// y (f32 [rows][cout]) = x16 (16-bit [rows][kp]) W^T + b, W host f32 [cout][cin].
bool linear_f32(p3d_ctx *ctx, const Buffer &x16, int64_t rows, int64_t kp, const float *w, const float *b, int cin,
                int cout, Buffer &y, std::string *error);
bool download_feats(p3d_ctx *ctx, const Buffer &y, std::size_t count, std::vector<float> &out, std::string *error);
// Multi-head attention on 16-bit rows [rows][heads*hd] (row pitches ld*,
// any even or odd hd <= 64); out16 gets [rows_q][ld_out] 16-bit rows
// (heads*hd columns, zero padding up to ld_out).
bool attention16(p3d_ctx *ctx, const void *q16, int64_t ldq, int64_t rows_q, const void *k16, int64_t ldk,
                 const void *v16, int64_t ldv, int64_t rows_k, const std::vector<int32_t> &cu_q,
                 const std::vector<int32_t> &cu_k, int heads, int hd, float scale, Buffer &out16, int64_t ld_out,
                 std::string *error);
// 16-bit [rows][heads*hd] (pitch ld) -> 16-bit [rows][heads*64].
bool heads_to_64(p3d_ctx *ctx, const void *x16, int64_t ld, int64_t rows, int heads, int hd, Buffer &out,
                 std::string *error);
// 16-bit [rows][ld] -> f32 [rows][cols] on the host.
bool operand_to_host(p3d_ctx *ctx, const void *x16, int64_t rows, int64_t cols, int64_t ld, std::vector<float> &out,
                     std::string *error);

// Device-side inputs of one transformer block.
struct BlockInputs {
    const Buffer *coords;            // int32 [n][4] (RoPE)
    std::vector<int32_t> offsets;    // batch offsets of the n rows
    int batch;
    int64_t n;
    const Buffer *ctx32;             // f32 [T][context_channels]
    const float *ctx_host;           // same values on the host (pitch padding path)
    std::vector<int32_t> ctx_offsets;
    const Buffer *proj32;            // f32 [n][proj_in] or null
    const float *proj_host;
};
// One block on the device, residual stream h (f32 [n][C]) updated in place;
// timestep_modulation: host [batch][6C].
bool block_device(p3d_ctx *ctx, Buffer &h, const BlockInputs &in, const float *timestep_modulation,
                  const SparseTransformerBlockConfig &config, const SparseTransformerBlockWeightsF32 &weights,
                  std::string *error);

}  // namespace b200
}  // namespace pixal3d
