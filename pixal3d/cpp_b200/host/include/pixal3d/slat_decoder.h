// SLat decoder (ConvNeXt levels joined by channel-to-spatial res blocks),
// B200 implementation with the reference's declarations
// (include/pixal3d/slat_decoder.h).  The whole decode runs in the
// device-resident p3d_decoder; the single-block functions run on the same
// kernels.  The mesh-extraction helpers of the reference header
// (dual_grid.h, SLatDecoderModel::decode_shape_mesh) are not part of this
// build.
#pragma once

#include <string>
#include <vector>

#include "pixal3d/sparse.h"

namespace pixal3d {

enum class SLatDecoderBlockKind {
    convnext,
    channel_to_spatial,
};

// Host f32 weights (borrowed).  Conv weights [27, out, in].
struct SLatDecoderBlockWeightsF32 {
    SLatDecoderBlockKind kind = SLatDecoderBlockKind::convnext;
    int channels = 0;
    int out_channels = 0;
    const float *norm_weight = nullptr;
    const float *norm_bias = nullptr;
    const float *norm1_weight = nullptr;
    const float *norm1_bias = nullptr;
    const float *conv1_weight = nullptr;
    const float *conv1_bias = nullptr;
    const float *norm2_weight = nullptr;
    const float *norm2_bias = nullptr;
    const float *conv2_weight = nullptr;
    const float *conv2_bias = nullptr;
    const float *mlp0_weight = nullptr;
    const float *mlp0_bias = nullptr;
    const float *mlp2_weight = nullptr;
    const float *mlp2_bias = nullptr;
    const float *to_subdiv_weight = nullptr;
    const float *to_subdiv_bias = nullptr;
    int mlp_hidden = 0;
};

constexpr float k_slat_decoder_final_layer_norm_eps = 1.0e-5f;

struct SLatDecoderConfig {
    int latent_channels = 0;
    int out_channels = 0;
    float norm_eps = 1e-6f;
    bool pred_subdiv = false;
    std::vector<int> model_channels;
    std::vector<int> num_blocks;
};

struct SLatDecoderWeightsF32 {
    const float *from_latent_weight = nullptr;
    const float *from_latent_bias = nullptr;
    const float *output_weight = nullptr;
    const float *output_bias = nullptr;
    std::vector<SLatDecoderBlockWeightsF32> blocks;
};

bool sparse_convnext_block_f32(const SparseTensorF32 &input, const SLatDecoderBlockWeightsF32 &weights,
                               float norm_eps, SparseTensorF32 &output, std::string *error = nullptr);

bool sparse_resblock_c2s_f32(const SparseTensorF32 &input, const SLatDecoderBlockWeightsF32 &weights, float norm_eps,
                             bool pred_subdiv, const SparseTensorF32 *subdivision, SparseTensorF32 &output,
                             SparseTensorF32 *predicted_subdiv = nullptr, std::string *error = nullptr);

bool slat_decoder_forward_f32(const SparseTensorF32 &input, const SLatDecoderConfig &config,
                              const SLatDecoderWeightsF32 &weights,
                              const std::vector<SparseTensorF32> *guide_subdivisions, SparseTensorF32 &output,
                              std::vector<SparseTensorF32> *predicted_subdivisions = nullptr,
                              std::string *error = nullptr);

bool slat_decoder_upsample_coords_f32(const SparseTensorF32 &input, const SLatDecoderConfig &config,
                                      const SLatDecoderWeightsF32 &weights, int upsample_times,
                                      SparseTensorF32 &output, std::string *error = nullptr);

struct SLatDecoderHParams {
    std::string component;
    std::string model_class;
    int resolution = 0;
    int latent_channels = 0;
    int out_channels = 0;
    float norm_eps = 1e-6f;
    bool pred_subdiv = false;
    std::vector<int> model_channels;
    std::vector<int> num_blocks;
};

class SLatDecoderModel {
public:
    SLatDecoderModel() = default;
    ~SLatDecoderModel();

    SLatDecoderModel(const SLatDecoderModel &) = delete;
    SLatDecoderModel &operator=(const SLatDecoderModel &) = delete;

    // Weight packs (GGUF) are not read by this build: returns false with a
    // message.  Use bind() with host weights instead.
    bool load(const std::string &path, const std::string &component, bool load_tensors = true,
              std::string *error = nullptr);
    // B200 extension: upload host f32 weights once (16-bit, device-resident).
    bool bind(const SLatDecoderHParams &hparams, const SLatDecoderWeightsF32 &weights, std::string *error = nullptr);
    void close() noexcept;

    bool is_loaded() const noexcept;
    bool has_data() const noexcept;
    const SLatDecoderHParams &hparams() const noexcept;
    int tensor_count() const noexcept;
    bool has_tensor(const std::string &name) const noexcept;

    bool decode(const SparseTensorF32 &input, const std::vector<SparseTensorF32> *guide_subdivisions,
                SparseTensorF32 &output, std::vector<SparseTensorF32> *predicted_subdivisions = nullptr,
                std::string *error = nullptr);
    bool upsample_coords(const SparseTensorF32 &input, int upsample_times, SparseTensorF32 &output,
                         std::string *error = nullptr);

private:
    struct Impl;
    Impl *impl_ = nullptr;
};

}  // namespace pixal3d
