// include/pixal3d/pipeline.h (SLat stages) on the B200 kernels:
// p3d_slat_normalize for the latent (de)normalization and
// p3d_quantize_slat_coords for the coordinate hand-off.
#include "pixal3d/pipeline.h"

#include <cmath>

#include "device.h"

namespace pixal3d {

using b200::Buffer;
using b200::fail;
using b200::ok;

namespace {

// valid_normalization (reference src/pipeline.cpp:268-285).
bool valid_normalization(const SLatNormalizationF32 &n, int channels, std::string *error) {
    if (channels <= 0 || n.mean.size() != static_cast<std::size_t>(channels) ||
        n.std.size() != static_cast<std::size_t>(channels))
        return fail(error, "SLat normalization channel count does not match model output");
    for (int c = 0; c < channels; ++c) {
        const float m = n.mean[static_cast<std::size_t>(c)], s = n.std[static_cast<std::size_t>(c)];
        if (!std::isfinite(m) || !std::isfinite(s) || s == 0.0f)
            return fail(error, "SLat normalization contains a non-finite or zero standard deviation");
    }
    return true;
}

// feats (host, [points][channels]) through p3d_slat_normalize, in place.
bool apply_normalization(SparseTensorF32 &t, const SLatNormalizationF32 &n, bool denormalize,
                         const char *nonfinite_message, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    const int64_t points = static_cast<int64_t>(t.points());
    if (points == 0) return true;
    Buffer x, mean, stdv;
    const std::size_t bytes = t.feats.size() * sizeof(float);
    if (!b200::upload(ctx, x, t.feats.data(), bytes, error) ||
        !b200::upload(ctx, mean, n.mean.data(), n.mean.size() * sizeof(float), error) ||
        !b200::upload(ctx, stdv, n.std.data(), n.std.size() * sizeof(float), error))
        return false;
    if (!ok(ctx, p3d_slat_normalize(ctx, x.as<float>(), points, t.channels, mean.as<float>(), stdv.as<float>(),
                                    denormalize ? 1 : 0, x.as<float>()),
            error))
        return false;
    const int rc = p3d_ctx_check(ctx);
    if (rc == P3D_ERR_NONFINITE) return fail(error, nonfinite_message);
    if (!ok(ctx, rc, error)) return false;
    return b200::download(ctx, t.feats.data(), x, bytes, error);
}

}  // namespace

bool normalize_slat_f32(const SparseTensorF32 &input, const SLatNormalizationF32 &normalization,
                        SparseTensorF32 &output, std::string *error) {
    output = SparseTensorF32{};
    if (!input.valid(error) || !valid_normalization(normalization, input.channels, error)) return false;
    SparseTensorF32 t = input;
    if (!apply_normalization(t, normalization, false, "SLat normalization produced a non-finite value", error))
        return false;
    output = std::move(t);
    return true;
}

bool run_slat_stage_f32(SLatFlowModel &flow_model, const SparseTensorF32 &noise,
                        const Pixal3DImageConditionF32 &condition, const FlowEulerSamplerConfig &sampler_config,
                        const SLatNormalizationF32 &normalization, SLatStageOutputF32 &output, std::string *error,
                        const SparseTensorF32 *concat_condition) {
    output = SLatStageOutputF32{};
    if (!flow_model.is_loaded() || !flow_model.has_data())
        return fail(error, "SLat flow model must be loaded with tensor data");
    if (!noise.valid(error) || !condition.global.valid(error) || (concat_condition && !concat_condition->valid(error)))
        return false;
    const SLatFlowHParams &hp = flow_model.hparams();
    if (noise.batch_size != condition.global.batch_size || condition.global.channels != hp.cond_channels ||
        condition.global.tokens() == 0)
        return fail(error, "SLat stage noise or global condition does not match model metadata");
    if (concat_condition) {
        const SparseTensorF32 &c = *concat_condition;
        if (c.batch_size != noise.batch_size || c.spatial_x != noise.spatial_x || c.spatial_y != noise.spatial_y ||
            c.spatial_z != noise.spatial_z || c.coords != noise.coords || c.channels <= 0 ||
            noise.channels + c.channels != hp.in_channels)
            return fail(error, "SLat stage concat condition does not match model input metadata");
    } else if (noise.channels != hp.in_channels) {
        return fail(error, "SLat stage noise channels do not match model input metadata");
    }
    const SparseTensorF32 *projection = nullptr;
    if (condition.has_projection()) {
        if (!condition.projection.valid(error) || condition.projection.batch_size != noise.batch_size ||
            condition.projection.coords != noise.coords)
            return fail(error, "SLat stage projection condition coordinates do not match noise");
        projection = &condition.projection;
    }
    if (hp.image_attn_mode == "proj" && (!projection || projection->channels != hp.proj_in_channels))
        return fail(error, "SLat stage projection condition is required by model metadata");
    if (!valid_normalization(normalization, hp.out_channels, error)) return false;
    if (!flow_model.sample(noise, sampler_config, condition.global, projection, output.flow, error, concat_condition))
        return false;
    output.latent = output.flow.samples;
    if (!apply_normalization(output.latent, normalization, true,
                             "SLat stage denormalization produced a non-finite value", error)) {
        output = SLatStageOutputF32{};
        return false;
    }
    return true;
}

bool quantize_slat_coords_f32(const SparseTensorF32 &upsampled_coords, int low_resolution, int requested_resolution,
                              std::size_t max_num_tokens, std::vector<std::int32_t> &coords, int &actual_resolution,
                              std::string *error) {
    coords.clear();
    actual_resolution = 0;
    if (!upsampled_coords.valid(error) || low_resolution <= 0)
        return fail(error, "invalid SLat cascade coordinate quantization input");
    if (requested_resolution != 1024) return fail(error, "SLat cascade resolution must be 1024");
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    const int64_t n = static_cast<int64_t>(upsampled_coords.points());
    const int batch = upsampled_coords.batch_size;
    Buffer dc, out, count, ws;
    const std::size_t wsb = p3d_quantize_slat_coords_workspace(batch);
    if ((n > 0 && !b200::upload(ctx, dc, upsampled_coords.coords.data(), static_cast<std::size_t>(n) * 16, error)) ||
        !out.allocate(ctx, static_cast<std::size_t>(n > 0 ? n : 1) * 16, error) || !count.allocate(ctx, 8, error) ||
        !ws.allocate(ctx, wsb, error))
        return false;
    if (!ok(ctx,
            p3d_quantize_slat_coords(ctx, dc.as<int32_t>(), n, batch, low_resolution, requested_resolution,
                                     out.as<int32_t>(), count.as<int64_t>(), ws.get(), wsb),
            error))
        return false;
    const int rc = p3d_ctx_check(ctx);
    if (rc == P3D_ERR_INVALID) return fail(error, "SLat decoder coordinate is outside cascade quantization range");
    if (!ok(ctx, rc, error)) return false;
    int64_t m = 0;
    if (!b200::download(ctx, &m, count, sizeof(m), error)) return false;
    if (max_num_tokens != 0 && static_cast<std::size_t>(m) > max_num_tokens)
        return fail(error, "quantized SLat coordinate count exceeds max_num_tokens at resolution 1024");
    coords.resize(static_cast<std::size_t>(m) * 4);
    if (m > 0 && !b200::download(ctx, coords.data(), out, coords.size() * 4, error)) return false;
    actual_resolution = 1024;
    return true;
}

}  // namespace pixal3d
