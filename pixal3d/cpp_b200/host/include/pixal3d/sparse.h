// Sparse-voxel tensors and operators of the SLat path, B200 implementation.
//
// Same declarations as the reference's include/pixal3d/sparse.h so callers
// compile unchanged; every operator runs on the GPU through the C ABI in
// p3d.h (host vectors are staged to device memory per call, operands are
// computed in f16 with f32 accumulation).  Errors: return false and set
// *error when non-null; the messages follow the reference's.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace pixal3d {

// Rows of `channels` features grouped into batch items by `offsets`
// (batch_size + 1 entries, offsets[0] = 0).
struct VarLenTensorF32 {
    int batch_size = 0;
    int channels = 0;
    std::vector<std::size_t> offsets;
    std::vector<float> feats;

    std::size_t tokens() const noexcept {
        return channels > 0 ? feats.size() / static_cast<std::size_t>(channels) : 0;
    }
    bool valid(std::string *error = nullptr) const;
};

// Active voxels: coords rows (batch, x, y, z), contiguous by batch, inside
// [0, batch_size) x [0, spatial_x) x [0, spatial_y) x [0, spatial_z);
// feats rows of `channels` values, one per voxel.
struct SparseTensorF32 {
    int batch_size = 0;
    int channels = 0;
    int spatial_x = 0;
    int spatial_y = 0;
    int spatial_z = 0;
    std::vector<std::int32_t> coords;
    std::vector<float> feats;

    std::size_t points() const noexcept { return coords.size() / 4; }
    bool valid(std::string *error = nullptr) const;
};

// y = W x + b per voxel, W row-major [out_channels, in_channels].
bool sparse_linear(const SparseTensorF32 &input, const float *weight, const float *bias, int out_channels,
                   SparseTensorF32 &output, std::string *error = nullptr);

bool varlen_linear(const VarLenTensorF32 &input, const float *weight, const float *bias, int out_channels,
                   VarLenTensorF32 &output, std::string *error = nullptr);

// LayerNorm over each voxel's channels; gamma and beta both null or both set.
bool sparse_layer_norm(const SparseTensorF32 &input, float epsilon, const float *gamma, const float *beta,
                       SparseTensorF32 &output, std::string *error = nullptr);

// Mean-pool into the grid divided by `factor`; output rows sorted by (b, x, y, z).
bool sparse_downsample_mean(const SparseTensorF32 &input, int factor, SparseTensorF32 &output,
                            std::string *error = nullptr);

// Move channel groups of factor^3 children into space; `subdivision` (same
// coords, factor^3 channels) keeps child c of a voxel where its value > 0.
bool sparse_channel_to_spatial(const SparseTensorF32 &input, int factor, const SparseTensorF32 *subdivision,
                               SparseTensorF32 &output, std::string *error = nullptr);

// Multi-head attention within each batch item.
bool sparse_scaled_dot_product_attention(const SparseTensorF32 &query, const SparseTensorF32 &key,
                                         const SparseTensorF32 &value, int num_heads, int head_dim, float scale,
                                         SparseTensorF32 &output, std::string *error = nullptr);

// Voxel queries attend to the variable-length key/value tokens of their batch item.
bool sparse_cross_attention(const SparseTensorF32 &query, const VarLenTensorF32 &key, const VarLenTensorF32 &value,
                            int num_heads, int head_dim, float scale, SparseTensorF32 &output,
                            std::string *error = nullptr);

// Interleaved-pair 3D rotary embedding from the voxel coordinates.
bool sparse_rotary_position_embedding(const SparseTensorF32 &input, int num_heads, int head_dim,
                                      float frequency_min, float frequency_base, SparseTensorF32 &output,
                                      std::string *error = nullptr);

// Per-head x / max(||x||, 1e-12) * sqrt(head_dim) * gamma.
bool sparse_multihead_rms_norm(const SparseTensorF32 &input, int num_heads, int head_dim, const float *gamma,
                               SparseTensorF32 &output, std::string *error = nullptr);

bool varlen_multihead_rms_norm(const VarLenTensorF32 &input, int num_heads, int head_dim, const float *gamma,
                               VarLenTensorF32 &output, std::string *error = nullptr);

// Submanifold 3x3x3 convolution, weight [27, out_channels, in_channels]
// with tap k = kd * 9 + kh * 3 + kw over offsets (kd-1, kh-1, kw-1).
bool sparse_submanifold_conv3d(const SparseTensorF32 &input, const float *weight, const float *bias,
                               int out_channels, SparseTensorF32 &output, std::string *error = nullptr);

}  // namespace pixal3d
