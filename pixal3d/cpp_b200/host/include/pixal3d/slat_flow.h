// SLat flow model (sparse-voxel flow transformer), B200 implementation with
// the reference's declarations (include/pixal3d/slat_flow.h).  The forward
// pass and the whole Euler/CFG sampling loop run on the GPU through
// p3d_flow_* (weights resident in 16-bit, one CUDA graph per step).
#pragma once

#include <cstddef>
#include <string>
#include <vector>

#include "pixal3d/flow_sampler.h"
#include "pixal3d/sparse_transformer.h"

namespace pixal3d {

struct SLatFlowHParams {
    std::string component;
    std::string model_class;
    int resolution = 0;
    int in_channels = 0;
    int out_channels = 0;
    int model_channels = 0;
    int cond_channels = 0;
    int num_blocks = 0;
    int num_heads = 0;
    int proj_in_channels = 0;
    float mlp_ratio = 0.0f;
    float norm_eps = 1e-6f;
    float rope_freq_min = 1.0f;
    float rope_freq_base = 10000.0f;
    std::string pe_mode = "rope";
    std::string image_attn_mode = "cross";
    bool share_mod = false;
    bool qk_rms_norm = false;
    bool qk_rms_norm_cross = false;

    int head_dim() const noexcept { return num_heads > 0 ? model_channels / num_heads : 0; }
};

// Host f32 weights in PyTorch [out, in] layout (borrowed).
struct SLatFlowWeightsF32 {
    const float *input_weight = nullptr;
    const float *input_bias = nullptr;
    const float *timestep_weight0 = nullptr;
    const float *timestep_bias0 = nullptr;
    const float *timestep_weight2 = nullptr;
    const float *timestep_bias2 = nullptr;
    const float *modulation_weight = nullptr;
    const float *modulation_bias = nullptr;
    const float *output_weight = nullptr;
    const float *output_bias = nullptr;
    std::vector<SparseTransformerBlockWeightsF32> blocks;
};

// One forward pass: input [N, in_channels] -> velocity [N, out_channels];
// timesteps one per batch item; global_context the condition tokens per
// item; projection_context [N, proj_in_channels] in proj mode.
bool slat_flow_forward_f32(const SparseTensorF32 &input, const float *timesteps, std::size_t timestep_count,
                           const VarLenTensorF32 &global_context, const SparseTensorF32 *projection_context,
                           const SLatFlowHParams &hparams, const SLatFlowWeightsF32 &weights, SparseTensorF32 &output,
                           std::string *error = nullptr, const SparseTensorF32 *concat_condition = nullptr);

class SLatFlowModel {
public:
    SLatFlowModel() = default;
    ~SLatFlowModel();

    SLatFlowModel(const SLatFlowModel &) = delete;
    SLatFlowModel &operator=(const SLatFlowModel &) = delete;

    // Load a component (shape_flow_512 / shape_flow_1024 / texture_flow_1024)
    // of a Pixal3D GGUF pack (compact-v1 tensor names; F32/F16/BF16); with
    // load_tensors the weights are uploaded to the device as by bind().
    bool load(const std::string &path, const std::string &component, bool load_tensors = true,
              std::string *error = nullptr);
    // B200 extension: upload host f32 weights once (16-bit, device-resident).
    bool bind(const SLatFlowHParams &hparams, const SLatFlowWeightsF32 &weights, std::string *error = nullptr);
    void close() noexcept;

    bool is_loaded() const noexcept;
    bool has_data() const noexcept;
    const SLatFlowHParams &hparams() const noexcept;
    int tensor_count() const noexcept;
    bool has_tensor(const std::string &name) const noexcept;

    bool forward(const SparseTensorF32 &input, const float *timesteps, std::size_t timestep_count,
                 const VarLenTensorF32 &global_context, const SparseTensorF32 *projection_context,
                 SparseTensorF32 &output, std::string *error = nullptr,
                 const SparseTensorF32 *concat_condition = nullptr);

    // Flow-Euler sampling with CFG against the zero condition (and zero
    // projection in proj mode), conditional and unconditional copies batched
    // on the device.
    bool sample(const SparseTensorF32 &noise, const FlowEulerSamplerConfig &sampler_config,
                const VarLenTensorF32 &global_context, const SparseTensorF32 *projection_context,
                FlowEulerSampleF32 &output, std::string *error = nullptr,
                const SparseTensorF32 *concat_condition = nullptr);

private:
public:
    struct Impl;  // defined by the implementation

private:
    Impl *impl_ = nullptr;
};

}  // namespace pixal3d
