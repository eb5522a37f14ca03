// SLat-stage part of the Pixal3D cascade (the reference's
// include/pixal3d/pipeline.h), B200 implementation.
//
// Same declarations as the reference for the SLat stages: the image
// condition container, latent normalization, one SLat stage (sampler +
// denormalization) and the decoder-coordinate quantization that hands the
// shape latent to the 1024 stages.  The sparse-structure stage, the full
// cascade driver and mesh extraction of the reference header are outside
// this library (they sit outside the SLat path).  Errors: return false and
// set *error, with the reference's messages.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "pixal3d/flow_sampler.h"
#include "pixal3d/slat_flow.h"
#include "pixal3d/sparse.h"

namespace pixal3d {

// Global tokens and (projection mode) per-voxel projected rows of one stage.
struct Pixal3DImageConditionF32 {
    VarLenTensorF32 global;
    SparseTensorF32 projection;

    bool has_projection() const noexcept { return projection.batch_size > 0 && projection.channels > 0; }
};

// Per-channel latent statistics: latent = normalized * std + mean.
struct SLatNormalizationF32 {
    std::vector<float> mean;
    std::vector<float> std;
};

// (latent - mean) / std, the representation a concat-conditioned flow reads.
bool normalize_slat_f32(const SparseTensorF32 &input, const SLatNormalizationF32 &normalization,
                        SparseTensorF32 &output, std::string *error = nullptr);

struct SLatStageOutputF32 {
    FlowEulerSampleF32 flow;
    SparseTensorF32 latent;
};

// Sample one SLat stage and denormalize its latent.
bool run_slat_stage_f32(SLatFlowModel &flow_model, const SparseTensorF32 &noise,
                        const Pixal3DImageConditionF32 &condition, const FlowEulerSamplerConfig &sampler_config,
                        const SLatNormalizationF32 &normalization, SLatStageOutputF32 &output,
                        std::string *error = nullptr, const SparseTensorF32 *concat_condition = nullptr);

// Decoder coordinates at low_resolution grid units -> unique coordinates on
// the 64^3 grid of the 1024 cascade (lexicographic order).  A non-zero
// max_num_tokens is a hard guard.
bool quantize_slat_coords_f32(const SparseTensorF32 &upsampled_coords, int low_resolution, int requested_resolution,
                              std::size_t max_num_tokens, std::vector<std::int32_t> &coords, int &actual_resolution,
                              std::string *error = nullptr);

}  // namespace pixal3d
