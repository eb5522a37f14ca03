// Flow-matching Euler sampler with classifier-free guidance, B200
// implementation with the reference's declarations
// (include/pixal3d/flow_sampler.h).  The CFG blend, guidance rescale and
// Euler update run on the GPU (p3d_euler_cfg_step).
#pragma once

#include <functional>
#include <string>
#include <vector>

#include "pixal3d/sparse.h"

namespace pixal3d {

struct FlowEulerSamplerConfig {
    int steps = 50;
    float sigma_min = 1e-5f;
    float rescale_t = 1.0f;
    float guidance_strength = 1.0f;
    float guidance_rescale = 0.0f;
    float guidance_interval_min = 0.0f;
    float guidance_interval_max = 1.0f;
    bool record_trajectory = false;
};

// Velocity model: fills `velocity` (same coords and channels as `state`) at
// model time 1000 * t, with the condition (true) or the null condition.
using FlowVelocityFn = std::function<bool(const SparseTensorF32 &state, float model_timestep, bool conditional,
                                          SparseTensorF32 &velocity, std::string *error)>;

struct FlowEulerSampleF32 {
    SparseTensorF32 samples;
    std::vector<SparseTensorF32> pred_x_t;
    std::vector<SparseTensorF32> pred_x_0;
};

bool flow_euler_sample_f32(const SparseTensorF32 &noise, const FlowEulerSamplerConfig &config,
                           const FlowVelocityFn &model, FlowEulerSampleF32 &output, std::string *error = nullptr);

}  // namespace pixal3d
