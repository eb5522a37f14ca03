// flow_euler_sample_f32, slat_flow_forward_f32 and SLatFlowModel on the B200
// kernels (src/flow_sampler.cpp:245-343, src/slat_flow.cpp:161-249,
// :1301-1447).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>

#include <map>
#include <memory>

#include "device.h"
#include "gguf.h"
#include "ops_internal.h"
#include "pixal3d/flow_sampler.h"
#include "pixal3d/slat_flow.h"

namespace pixal3d {

using b200::Buffer;
using b200::fail;
using b200::ok;

namespace {

bool valid_config(const FlowEulerSamplerConfig &c, std::string *error) {
    if (c.steps <= 0 || !(c.sigma_min >= 0.0f) || !(c.sigma_min < 1.0f) || !std::isfinite(c.sigma_min) ||
        !(c.rescale_t > 0.0f) || !std::isfinite(c.rescale_t) || !std::isfinite(c.guidance_strength) ||
        !std::isfinite(c.guidance_rescale) || c.guidance_rescale < 0.0f || !std::isfinite(c.guidance_interval_min) ||
        !std::isfinite(c.guidance_interval_max) || c.guidance_interval_min > c.guidance_interval_max)
        return fail(error, "invalid flow Euler sampler configuration");
    return true;
}

bool same_layout(const SparseTensorF32 &a, const SparseTensorF32 &b) {
    return a.batch_size == b.batch_size && a.channels == b.channels && a.spatial_x == b.spatial_x &&
           a.spatial_y == b.spatial_y && a.spatial_z == b.spatial_z && a.coords == b.coords;
}

// t_i = r l / (1 + (r - 1) l), l = 1 - i / steps (src/flow_sampler.cpp:268-286)
bool schedule(const FlowEulerSamplerConfig &c, int step, float &t, std::string *error) {
    const float lin = 1.0f - static_cast<float>(step) / static_cast<float>(c.steps);
    const float den = 1.0f + (c.rescale_t - 1.0f) * lin;
    if (!(den > 0.0f) || !std::isfinite(den)) return fail(error, "flow Euler timestep schedule is not finite");
    t = c.rescale_t * lin / den;
    return true;
}

}  // namespace

bool flow_euler_sample_f32(const SparseTensorF32 &noise, const FlowEulerSamplerConfig &config,
                           const FlowVelocityFn &model, FlowEulerSampleF32 &output, std::string *error) {
    output = FlowEulerSampleF32{};
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer x;
    if (!b200::validate_sparse(ctx, noise, nullptr, &x, error) || !valid_config(config, error)) return false;
    if (!model) return fail(error, "flow Euler sampler model callback is empty");
    SparseTensorF32 state = noise;
    const int64_t n = static_cast<int64_t>(state.points());
    const int ch = state.channels;
    const std::size_t count = static_cast<std::size_t>(n) * ch;
    const std::vector<int32_t> offs = b200::batch_offsets(state);
    Buffer doffs, stats, vp, vn, x0;
    if (!b200::upload(ctx, doffs, offs.data(), offs.size() * 4, error) ||
        !stats.allocate(ctx, sizeof(double) * 4 * state.batch_size, error) ||
        !vp.allocate(ctx, count * 4, error) || !vn.allocate(ctx, count * 4, error) ||
        (config.record_trajectory && !x0.allocate(ctx, count * 4, error)))
        return false;
    SparseTensorF32 positive, negative;
    for (int step = 0; step < config.steps; ++step) {
        float t = 0.0f, tn = 0.0f;
        if (!schedule(config, step, t, error) || !schedule(config, step + 1, tn, error)) return false;
        const bool in_interval = t >= config.guidance_interval_min && t <= config.guidance_interval_max;
        const float guidance = in_interval ? config.guidance_strength : 1.0f;
        const bool cfg = guidance != 1.0f && guidance != 0.0f;
        // guidance 1: conditional only; 0: unconditional only; else both + blend
        if (!model(state, 1000.0f * t, guidance != 0.0f, positive, error)) return false;
        if (!positive.valid(error)) return false;
        if (!same_layout(state, positive))
            return fail(error, "flow model velocity shape or coordinates changed during sampling");
        if (cfg) {
            if (!model(state, 1000.0f * t, false, negative, error)) return false;
            if (!negative.valid(error)) return false;
            if (!same_layout(state, negative))
                return fail(error, "flow model velocity shape or coordinates changed during sampling");
        }
        if (!ok(ctx, p3d_copy_to_device(ctx, vp.get(), positive.feats.data(), count * 4), error) ||
            (cfg && !ok(ctx, p3d_copy_to_device(ctx, vn.get(), negative.feats.data(), count * 4), error)))
            return false;
        const float gr = cfg ? config.guidance_rescale : 0.0f;
        if (n > 0 && !ok(ctx,
                         p3d_euler_cfg_step(ctx, x.as<float>(), vp.as<float>(), cfg ? vn.as<float>() : nullptr, n, ch,
                                            doffs.as<int32_t>(), state.batch_size, t, tn, cfg ? guidance : 1.0f, gr,
                                            config.sigma_min, stats.as<double>(),
                                            config.record_trajectory ? x0.as<float>() : nullptr),
                         error))
            return false;
        if (!b200::download(ctx, state.feats.data(), x, count * 4, error)) return false;
        if (config.record_trajectory) {
            SparseTensorF32 pred0 = state;
            if (!b200::download(ctx, pred0.feats.data(), x0, count * 4, error)) return false;
            output.pred_x_t.push_back(state);
            output.pred_x_0.push_back(std::move(pred0));
        }
    }
    output.samples = std::move(state);
    return true;
}

// ------------------------------------------------------------ flow model

namespace {

struct DeviceWeights {
    std::vector<Buffer> bufs;
    std::vector<p3d_block_weights> blocks;
    p3d_flow_weights w{};
    const float *put(p3d_ctx *ctx, const float *host, std::size_t count, bool &okay, std::string *error) {
        if (!host || !okay) return nullptr;
        bufs.emplace_back();
        okay = b200::upload(ctx, bufs.back(), host, count * sizeof(float), error);
        return bufs.back().as<float>();
    }
};

bool to_hparams(const SLatFlowHParams &h, p3d_flow_hparams &out, std::string *error) {
    std::memset(&out, 0, sizeof(out));
    if (h.model_channels <= 0 || h.num_heads <= 0 || h.num_blocks <= 0 || h.in_channels <= 0 ||
        h.out_channels <= 0 || h.cond_channels <= 0 || !(h.mlp_ratio > 0.0f) || h.model_channels % h.num_heads != 0)
        return fail(error, "invalid SLat flow hyperparameters");
    if (h.pe_mode != "rope" && h.pe_mode != "ape") return fail(error, "unsupported SLat flow pe_mode");
    if (h.image_attn_mode != "cross" && h.image_attn_mode != "proj")
        return fail(error, "unsupported SLat flow image_attn_mode");
    out.in_channels = h.in_channels;
    out.out_channels = h.out_channels;
    out.model_channels = h.model_channels;
    out.cond_channels = h.cond_channels;
    out.num_blocks = h.num_blocks;
    out.num_heads = h.num_heads;
    out.mlp_hidden = static_cast<int>(static_cast<float>(h.model_channels) * h.mlp_ratio);
    out.proj_in_channels = h.proj_in_channels;
    out.proj_mode = h.image_attn_mode == "proj" ? 1 : 0;
    out.qk_rms_norm = h.qk_rms_norm ? 1 : 0;
    out.qk_rms_norm_cross = h.qk_rms_norm_cross ? 1 : 0;
    out.pe_mode = h.pe_mode == "ape" ? 1 : 0;
    out.io_resblocks = 0;
    out.groups = 32;
    out.operand_dtype = b200::kOperand;
    out.norm_eps = h.norm_eps;
    out.rope_freq_min = h.rope_freq_min;
    out.rope_freq_base = h.rope_freq_base;
    return true;
}

// Upload host weights and build the device-resident flow (16-bit copies);
// the f32 staging buffers are released when this returns.
bool create_flow(p3d_ctx *ctx, const SLatFlowHParams &h, const SLatFlowWeightsF32 &w, p3d_flow **flow,
                 std::string *error) {
    p3d_flow_hparams hp;
    if (!to_hparams(h, hp, error)) return false;
    if (static_cast<int>(w.blocks.size()) != h.num_blocks) return fail(error, "SLat flow block count mismatch");
    const std::size_t C = h.model_channels, mlp = hp.mlp_hidden, cc = h.cond_channels, pin = h.proj_in_channels;
    DeviceWeights d;
    bool okay = true;
    d.w.input_w = d.put(ctx, w.input_weight, C * h.in_channels, okay, error);
    d.w.input_b = d.put(ctx, w.input_bias, C, okay, error);
    d.w.t_w0 = d.put(ctx, w.timestep_weight0, C * 256, okay, error);
    d.w.t_b0 = d.put(ctx, w.timestep_bias0, C, okay, error);
    d.w.t_w2 = d.put(ctx, w.timestep_weight2, C * C, okay, error);
    d.w.t_b2 = d.put(ctx, w.timestep_bias2, C, okay, error);
    d.w.mod_w = d.put(ctx, w.modulation_weight, 6 * C * C, okay, error);
    d.w.mod_b = d.put(ctx, w.modulation_bias, 6 * C, okay, error);
    d.w.output_w = d.put(ctx, w.output_weight, C * h.out_channels, okay, error);
    d.w.output_b = d.put(ctx, w.output_bias, h.out_channels, okay, error);
    d.bufs.reserve(d.bufs.size() + 24 * w.blocks.size());
    for (const SparseTransformerBlockWeightsF32 &b : w.blocks) {
        p3d_block_weights o{};
        o.modulation = d.put(ctx, b.modulation, 6 * C, okay, error);
        o.qkv_w = d.put(ctx, b.self_to_qkv_weight, 3 * C * C, okay, error);
        o.qkv_b = d.put(ctx, b.self_to_qkv_bias, 3 * C, okay, error);
        o.q_gamma = d.put(ctx, b.self_q_gamma, C, okay, error);
        o.k_gamma = d.put(ctx, b.self_k_gamma, C, okay, error);
        o.out_w = d.put(ctx, b.self_to_out_weight, C * C, okay, error);
        o.out_b = d.put(ctx, b.self_to_out_bias, C, okay, error);
        o.norm2_w = d.put(ctx, b.norm2_weight, C, okay, error);
        o.norm2_b = d.put(ctx, b.norm2_bias, C, okay, error);
        o.cq_w = d.put(ctx, b.cross_to_q_weight, C * C, okay, error);
        o.cq_b = d.put(ctx, b.cross_to_q_bias, C, okay, error);
        o.ckv_w = d.put(ctx, b.cross_to_kv_weight, 2 * C * cc, okay, error);
        o.ckv_b = d.put(ctx, b.cross_to_kv_bias, 2 * C, okay, error);
        o.cq_gamma = d.put(ctx, b.cross_q_gamma, C, okay, error);
        o.ck_gamma = d.put(ctx, b.cross_k_gamma, C, okay, error);
        o.co_w = d.put(ctx, b.cross_to_out_weight, C * C, okay, error);
        o.co_b = d.put(ctx, b.cross_to_out_bias, C, okay, error);
        o.proj_w = d.put(ctx, b.proj_weight, C * pin, okay, error);
        o.proj_b = d.put(ctx, b.proj_bias, C, okay, error);
        o.mlp0_w = d.put(ctx, b.mlp0_weight, mlp * C, okay, error);
        o.mlp0_b = d.put(ctx, b.mlp0_bias, mlp, okay, error);
        o.mlp2_w = d.put(ctx, b.mlp2_weight, C * mlp, okay, error);
        o.mlp2_b = d.put(ctx, b.mlp2_bias, C, okay, error);
        d.blocks.push_back(o);
    }
    if (!okay) return false;
    d.w.blocks = d.blocks.data();
    return ok(ctx, p3d_flow_create(ctx, &hp, &d.w, flow), error);
}

// Bind the input's coordinates (as `copies` stacked copies, copy j's batch
// items shifted by j * batch_size) and the condition offsets.
bool prepare(p3d_ctx *ctx, p3d_flow *flow, const SparseTensorF32 &input, int copies,
             const std::vector<int64_t> &ctx_offsets, Buffer &coords, std::string *error) {
    const std::size_t n = input.points();
    std::vector<int32_t> c(n * 4 * copies);
    for (int j = 0; j < copies; ++j)
        for (std::size_t p = 0; p < n; ++p) {
            c[(j * n + p) * 4] = input.coords[p * 4] + j * input.batch_size;
            for (int a = 1; a < 4; ++a) c[(j * n + p) * 4 + a] = input.coords[p * 4 + a];
        }
    if (!b200::upload(ctx, coords, c.data(), c.size() * 4, error)) return false;
    return ok(ctx,
              p3d_flow_prepare(flow, coords.as<int32_t>(), static_cast<int64_t>(n) * copies,
                               input.batch_size * copies, input.spatial_x, input.spatial_y, input.spatial_z,
                               ctx_offsets.data()),
              error);
}

// concat_sparse_features (src/slat_flow.cpp:50-75): rows [left | right]
// with the same coordinates; a host row copy of the API's host tensors.
bool concat_features(const SparseTensorF32 &left, const SparseTensorF32 &right, SparseTensorF32 &out,
                     std::string *error) {
    if (left.batch_size != right.batch_size || left.spatial_x != right.spatial_x ||
        left.spatial_y != right.spatial_y || left.spatial_z != right.spatial_z || left.coords != right.coords ||
        right.channels <= 0 || left.channels > std::numeric_limits<int>::max() - right.channels ||
        right.feats.size() != right.points() * static_cast<std::size_t>(right.channels))
        return fail(error, "SLat flow concat condition shape or coordinates mismatch");
    out = left;
    out.channels = left.channels + right.channels;
    const std::size_t n = left.points(), lc = static_cast<std::size_t>(left.channels),
                      rc = static_cast<std::size_t>(right.channels);
    out.feats.resize(n * (lc + rc));
    for (std::size_t p = 0; p < n; ++p) {
        std::copy(left.feats.begin() + static_cast<std::ptrdiff_t>(p * lc),
                  left.feats.begin() + static_cast<std::ptrdiff_t>((p + 1) * lc),
                  out.feats.begin() + static_cast<std::ptrdiff_t>(p * (lc + rc)));
        std::copy(right.feats.begin() + static_cast<std::ptrdiff_t>(p * rc),
                  right.feats.begin() + static_cast<std::ptrdiff_t>((p + 1) * rc),
                  out.feats.begin() + static_cast<std::ptrdiff_t>(p * (lc + rc) + lc));
    }
    return true;
}

bool check_forward_inputs(const SparseTensorF32 &input, std::size_t timestep_count,
                          const VarLenTensorF32 &global_context, const SparseTensorF32 *projection_context,
                          const SLatFlowHParams &h, const SparseTensorF32 *concat_condition, std::string *error) {
    if (concat_condition &&
        (concat_condition->batch_size != input.batch_size || concat_condition->spatial_x != input.spatial_x ||
         concat_condition->spatial_y != input.spatial_y || concat_condition->spatial_z != input.spatial_z ||
         concat_condition->coords != input.coords || concat_condition->channels <= 0))
        return fail(error, "SLat flow concat condition shape or coordinates mismatch");
    const int in_channels = input.channels + (concat_condition ? concat_condition->channels : 0);
    if (in_channels != h.in_channels || global_context.channels != h.cond_channels ||
        global_context.batch_size != input.batch_size || timestep_count != static_cast<std::size_t>(input.batch_size))
        return fail(error, "SLat flow input, timestep or context shape mismatch");
    if (h.image_attn_mode == "proj" &&
        (!projection_context || projection_context->channels != h.proj_in_channels ||
         projection_context->coords != input.coords))
        return fail(error, "SLat flow projection context shape mismatch");
    return true;
}

bool run_forward(p3d_ctx *ctx, p3d_flow *flow, const SparseTensorF32 &input, const float *timesteps,
                 const VarLenTensorF32 &global_context, const SparseTensorF32 *projection_context,
                 const SLatFlowHParams &h, SparseTensorF32 &output, std::string *error) {
    Buffer x, g, coords, ts, proj, y;
    if (!b200::validate_sparse(ctx, input, nullptr, &x, error) ||
        !b200::validate_varlen(ctx, global_context, &g, error))
        return false;
    if (h.image_attn_mode == "proj" && !b200::validate_sparse(ctx, *projection_context, nullptr, &proj, error))
        return false;
    std::vector<int64_t> coff(global_context.offsets.begin(), global_context.offsets.end());
    if (!prepare(ctx, flow, input, 1, coff, coords, error) ||
        !b200::upload(ctx, ts, timesteps, sizeof(float) * input.batch_size, error))
        return false;
    const std::size_t count = input.points() * static_cast<std::size_t>(h.out_channels);
    if (!y.allocate(ctx, count * 4, error)) return false;
    if (!ok(ctx,
            p3d_flow_forward(flow, x.as<float>(), ts.as<float>(), g.get(), P3D_F32,
                             h.image_attn_mode == "proj" ? proj.as<float>() : nullptr, y.as<float>()),
            error))
        return false;
    std::vector<float> feats;
    if (!b200::download_feats(ctx, y, count, feats, error)) return false;
    b200::copy_shape(input, h.out_channels, output);
    output.feats = std::move(feats);
    return true;
}

// The device-resident model (p3d_flow) covers model_channels % 64 == 0 with
// 64-wide heads and mlp_hidden % 8 == 0 (every Pixal3D SLat model).  Other
// shapes run the same forward composed from the per-operator kernels.
bool device_flow_supported(const SLatFlowHParams &h) {
    const int mlp = static_cast<int>(static_cast<float>(h.model_channels) * h.mlp_ratio);
    return h.num_heads > 0 && h.model_channels % 64 == 0 && h.model_channels / h.num_heads == 64 && mlp % 8 == 0;
}

bool composed_forward(p3d_ctx *ctx, const SparseTensorF32 &input, const float *timesteps,
                      const VarLenTensorF32 &global_context, const SparseTensorF32 *projection_context,
                      const SLatFlowHParams &h, const SLatFlowWeightsF32 &w, SparseTensorF32 &output,
                      std::string *error) {
    if (h.pe_mode != "rope") return fail(error, "SLat flow pe_mode other than rope needs model_channels % 64 == 0");
    if (static_cast<int>(w.blocks.size()) != h.num_blocks) return fail(error, "SLat flow block count mismatch");
    const bool proj = h.image_attn_mode == "proj";
    Buffer c32, x32, g32, p32;
    if (!b200::validate_sparse(ctx, input, &c32, &x32, error) || !b200::validate_varlen(ctx, global_context, &g32, error))
        return false;
    if (proj && !b200::validate_sparse(ctx, *projection_context, nullptr, &p32, error)) return false;
    const int C = h.model_channels, B = input.batch_size;
    const int64_t n = static_cast<int64_t>(input.points());
    if (!w.timestep_weight0 || !w.timestep_bias0 || !w.timestep_weight2 || !w.timestep_bias2 ||
        !w.modulation_weight || !w.modulation_bias || !w.input_weight || !w.output_weight)
        return fail(error, "missing SLat flow tensor");
    // timestep conditioning -> per-item 6C modulation (device), read back for the blocks
    Buffer ts, tw0, tb0, tw2, tb2, mw, mb, scratch, tmod;
    if (!b200::upload(ctx, ts, timesteps, sizeof(float) * B, error) ||
        !b200::upload(ctx, tw0, w.timestep_weight0, sizeof(float) * C * 256, error) ||
        !b200::upload(ctx, tb0, w.timestep_bias0, sizeof(float) * C, error) ||
        !b200::upload(ctx, tw2, w.timestep_weight2, sizeof(float) * C * C, error) ||
        !b200::upload(ctx, tb2, w.timestep_bias2, sizeof(float) * C, error) ||
        !b200::upload(ctx, mw, w.modulation_weight, sizeof(float) * 6 * C * C, error) ||
        !b200::upload(ctx, mb, w.modulation_bias, sizeof(float) * 6 * C, error) ||
        !scratch.allocate(ctx, sizeof(float) * B * (256 + 2 * C), error) ||
        !tmod.allocate(ctx, sizeof(float) * B * 6 * C, error))
        return false;
    if (!ok(ctx,
            p3d_timestep_mlp(ctx, ts.as<float>(), B, C, tw0.as<float>(), tb0.as<float>(), tw2.as<float>(),
                             tb2.as<float>(), mw.as<float>(), mb.as<float>(), scratch.as<float>(), tmod.as<float>()),
            error))
        return false;
    std::vector<float> tmod_h(static_cast<std::size_t>(B) * 6 * C);
    if (!b200::download(ctx, tmod_h.data(), tmod, tmod_h.size() * 4, error)) return false;
    // input linear into the f32 residual stream
    const int64_t in_pad = b200::round_up(h.in_channels, 8);
    Buffer x16, hs;
    if (!b200::to_operand(ctx, x32, input.feats.data(), n, h.in_channels, in_pad, x16, error) ||
        !b200::linear_f32(ctx, x16, n, in_pad, w.input_weight, w.input_bias, h.in_channels, C, hs, error))
        return false;
    SparseTransformerBlockConfig cfg;
    cfg.channels = C;
    cfg.num_heads = h.num_heads;
    cfg.mlp_hidden = static_cast<int>(static_cast<float>(C) * h.mlp_ratio);
    cfg.context_channels = h.cond_channels;
    cfg.proj_in_channels = h.proj_in_channels;
    cfg.norm_eps = h.norm_eps;
    cfg.rope_freq_min = h.rope_freq_min;
    cfg.rope_freq_base = h.rope_freq_base;
    cfg.use_rope = true;
    cfg.qk_rms_norm = h.qk_rms_norm;
    cfg.qk_rms_norm_cross = h.qk_rms_norm_cross;
    cfg.use_projection = proj;
    b200::BlockInputs in{&c32, b200::batch_offsets(input), B, n, &g32, global_context.feats.data(),
                         b200::varlen_offsets(global_context), proj ? &p32 : nullptr,
                         proj ? projection_context->feats.data() : nullptr};
    for (const SparseTransformerBlockWeightsF32 &bw : w.blocks)
        if (!b200::block_device(ctx, hs, in, tmod_h.data(), cfg, bw, error)) return false;
    // final LayerNorm (eps 1e-5, src/slat_flow.cpp:244-248) + output linear
    const int64_t Cp = b200::round_up(C, 8);
    Buffer xn, xnp, y;
    if (!xn.allocate(ctx, static_cast<std::size_t>(n) * C * 2, error)) return false;
    if (n > 0 && !ok(ctx,
                     p3d_layernorm_modulate(ctx, hs.as<float>(), n, C, 1e-5f, nullptr, nullptr, nullptr, 0, nullptr, 0,
                                            xn.get(), b200::kOperand),
                     error))
        return false;
    const Buffer *xo = &xn;
    if (Cp != C) {
        if (!xnp.allocate(ctx, static_cast<std::size_t>(n) * Cp * 2, error)) return false;
        if (n > 0 && !ok(ctx, p3d_repack_heads(ctx, xn.get(), C, n, 1, C, C, xnp.get(), Cp, b200::kOperand), error))
            return false;
        xo = &xnp;
    }
    if (!b200::linear_f32(ctx, *xo, n, Cp, w.output_weight, w.output_bias, C, h.out_channels, y, error)) return false;
    std::vector<float> feats;
    if (!b200::download_feats(ctx, y, static_cast<std::size_t>(n) * h.out_channels, feats, error)) return false;
    b200::copy_shape(input, h.out_channels, output);
    output.feats = std::move(feats);
    return true;
}

// Owned copies of a model's host weights (for the composed path).
struct HostWeights {
    std::vector<std::vector<float>> store;
    SLatFlowWeightsF32 w;
    const float *keep(const float *p, std::size_t count) {
        if (!p) return nullptr;
        store.emplace_back(p, p + count);
        return store.back().data();
    }
    void copy(const SLatFlowHParams &h, const SLatFlowWeightsF32 &src) {
        const std::size_t C = h.model_channels, mlp = static_cast<std::size_t>(static_cast<float>(C) * h.mlp_ratio);
        const std::size_t cc = h.cond_channels, pin = h.proj_in_channels;
        store.reserve(10 + 23 * src.blocks.size());
        w.input_weight = keep(src.input_weight, C * h.in_channels);
        w.input_bias = keep(src.input_bias, C);
        w.timestep_weight0 = keep(src.timestep_weight0, C * 256);
        w.timestep_bias0 = keep(src.timestep_bias0, C);
        w.timestep_weight2 = keep(src.timestep_weight2, C * C);
        w.timestep_bias2 = keep(src.timestep_bias2, C);
        w.modulation_weight = keep(src.modulation_weight, 6 * C * C);
        w.modulation_bias = keep(src.modulation_bias, 6 * C);
        w.output_weight = keep(src.output_weight, C * h.out_channels);
        w.output_bias = keep(src.output_bias, h.out_channels);
        for (const SparseTransformerBlockWeightsF32 &b : src.blocks) {
            SparseTransformerBlockWeightsF32 o;
            o.modulation = keep(b.modulation, 6 * C);
            o.self_to_qkv_weight = keep(b.self_to_qkv_weight, 3 * C * C);
            o.self_to_qkv_bias = keep(b.self_to_qkv_bias, 3 * C);
            o.self_q_gamma = keep(b.self_q_gamma, C);
            o.self_k_gamma = keep(b.self_k_gamma, C);
            o.self_to_out_weight = keep(b.self_to_out_weight, C * C);
            o.self_to_out_bias = keep(b.self_to_out_bias, C);
            o.norm2_weight = keep(b.norm2_weight, C);
            o.norm2_bias = keep(b.norm2_bias, C);
            o.cross_to_q_weight = keep(b.cross_to_q_weight, C * C);
            o.cross_to_q_bias = keep(b.cross_to_q_bias, C);
            o.cross_to_kv_weight = keep(b.cross_to_kv_weight, 2 * C * cc);
            o.cross_to_kv_bias = keep(b.cross_to_kv_bias, 2 * C);
            o.cross_q_gamma = keep(b.cross_q_gamma, C);
            o.cross_k_gamma = keep(b.cross_k_gamma, C);
            o.cross_to_out_weight = keep(b.cross_to_out_weight, C * C);
            o.cross_to_out_bias = keep(b.cross_to_out_bias, C);
            o.proj_weight = keep(b.proj_weight, C * pin);
            o.proj_bias = keep(b.proj_bias, C);
            o.mlp0_weight = keep(b.mlp0_weight, mlp * C);
            o.mlp0_bias = keep(b.mlp0_bias, mlp);
            o.mlp2_weight = keep(b.mlp2_weight, C * mlp);
            o.mlp2_bias = keep(b.mlp2_bias, C);
            w.blocks.push_back(o);
        }
    }
};

}  // namespace

bool slat_flow_forward_f32(const SparseTensorF32 &input, const float *timesteps, std::size_t timestep_count,
                           const VarLenTensorF32 &global_context, const SparseTensorF32 *projection_context,
                           const SLatFlowHParams &hparams, const SLatFlowWeightsF32 &weights, SparseTensorF32 &output,
                           std::string *error, const SparseTensorF32 *concat_condition) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    if (!timesteps) return fail(error, "SLat flow timesteps are null");
    if (!check_forward_inputs(input, timestep_count, global_context, projection_context, hparams, concat_condition,
                              error))
        return false;
    SparseTensorF32 joined;
    if (concat_condition && !concat_features(input, *concat_condition, joined, error)) return false;
    const SparseTensorF32 &model_input = concat_condition ? joined : input;
    if (!device_flow_supported(hparams))
        return composed_forward(ctx, model_input, timesteps, global_context, projection_context, hparams, weights,
                                output, error);
    p3d_flow *flow = nullptr;
    if (!create_flow(ctx, hparams, weights, &flow, error)) return false;
    const bool r =
        run_forward(ctx, flow, model_input, timesteps, global_context, projection_context, hparams, output, error);
    p3d_flow_destroy(flow);
    return r;
}

struct SLatFlowModel::Impl {
    SLatFlowHParams hp;
    p3d_flow *flow = nullptr;  // device-resident model, or
    HostWeights host;          // weights for the composed path
    int tensors = 0;
    bool has_data = true;
    std::string alias;                                 // pack component prefix (load())
    std::vector<std::string> pack_tensors;             // this component's tensor names in the pack
    std::map<std::string, std::vector<float>> values;  // loaded tensors, f32
    ~Impl() {
        if (flow) p3d_flow_destroy(flow);
    }
};

namespace {

// Component name -> tensor-name prefix of the compact-v1 pack scheme
// (compact_prefix, src/slat_flow.cpp:353-358).
std::string compact_prefix(const std::string &component) {
    if (component == "shape_flow_512") return "sh512";
    if (component == "shape_flow_1024") return "sh1024";
    if (component == "texture_flow_1024") return "tx1024";
    return {};
}

bool starts_with(const std::string &s, const std::string &p) { return s.size() >= p.size() && s.compare(0, p.size(), p) == 0; }

// Hyperparameters under "pixal3d.<component>." (read_hparams,
// src/slat_flow.cpp:397-427): the integer and mlp_ratio keys are required,
// the rest optional with the reference's defaults.
bool read_flow_hparams(const b200::GgufFile &f, const std::string &component, SLatFlowHParams &hp,
                       std::string *error) {
    const std::string k = "pixal3d." + component + ".";
    uint32_t v = 0;
    if (!f.get_string(k + "model_class", hp.model_class, true, error)) return false;
    struct IntKey {
        const char *name;
        int *dst;
    } ints[] = {{"resolution", &hp.resolution},         {"in_channels", &hp.in_channels},
                {"out_channels", &hp.out_channels},     {"model_channels", &hp.model_channels},
                {"cond_channels", &hp.cond_channels},   {"num_blocks", &hp.num_blocks},
                {"num_heads", &hp.num_heads}};
    for (const IntKey &ik : ints) {
        if (!f.get_u32(k + ik.name, v, true, error)) return false;
        *ik.dst = static_cast<int>(v);
    }
    v = 0;
    if (!f.get_f32(k + "mlp_ratio", hp.mlp_ratio, true, error) ||
        !f.get_string(k + "pe_mode", hp.pe_mode, false, error) ||
        !f.get_bool(k + "share_mod", hp.share_mod, false, error) ||
        !f.get_bool(k + "qk_rms_norm", hp.qk_rms_norm, false, error) ||
        !f.get_bool(k + "qk_rms_norm_cross", hp.qk_rms_norm_cross, false, error) ||
        !f.get_f32(k + "rope_freq_min", hp.rope_freq_min, false, error) ||
        !f.get_f32(k + "rope_freq_base", hp.rope_freq_base, false, error) ||
        !f.get_string(k + "image_attn_mode", hp.image_attn_mode, false, error) ||
        !f.get_u32(k + "proj_in_channels", v, false, error))
        return false;
    if (hp.pe_mode.empty()) hp.pe_mode = "rope";
    if (hp.image_attn_mode.empty()) hp.image_attn_mode = "cross";
    hp.proj_in_channels = v == 0 ? hp.cond_channels : static_cast<int>(v);
    // the reference's valid_hparams (src/slat_flow.cpp:113-138)
    if (hp.resolution <= 0 || hp.in_channels <= 0 || hp.out_channels <= 0 || hp.model_channels <= 0 ||
        hp.cond_channels <= 0 || hp.num_blocks <= 0 || hp.num_heads <= 0 || hp.model_channels % hp.num_heads != 0 ||
        hp.head_dim() % 2 != 0 || !(hp.mlp_ratio > 0.0f) || !std::isfinite(hp.mlp_ratio) ||
        !(hp.rope_freq_min > 0.0f) || !(hp.rope_freq_base > 0.0f) || !std::isfinite(hp.rope_freq_min) ||
        !std::isfinite(hp.rope_freq_base))
        return fail(error, "invalid SLat flow hyperparameters");
    if (hp.pe_mode != "rope" || !hp.share_mod)
        return fail(error, "SLat flow currently requires pe_mode=rope and share_mod=true");
    if (hp.image_attn_mode != "cross" && hp.image_attn_mode != "proj")
        return fail(error, "SLat flow supports image_attn_mode cross or proj");
    if (hp.image_attn_mode == "proj" && hp.proj_in_channels <= 0)
        return fail(error, "SLat flow projection channels must be positive");
    return true;
}

// Weight pointers into the loaded tensors, each checked for its element
// count (the names of SLatFlowModel::forward, src/slat_flow.cpp:1347-1393).
bool pack_weights(const SLatFlowModel::Impl &m, SLatFlowWeightsF32 &w, std::string *error);

}  // namespace

SLatFlowModel::~SLatFlowModel() { close(); }

void SLatFlowModel::close() noexcept {
    delete impl_;
    impl_ = nullptr;
}

namespace {
bool pack_weights(const SLatFlowModel::Impl &m, SLatFlowWeightsF32 &w, std::string *error) {
    const SLatFlowHParams &h = m.hp;
    const std::size_t C = h.model_channels, mlp = static_cast<std::size_t>(static_cast<float>(C) * h.mlp_ratio);
    const std::size_t cc = h.cond_channels, pin = h.proj_in_channels;
    bool okay = true;
    // required tensor of `count` elements (optional: nullptr when absent)
    auto get = [&](const std::string &local, std::size_t count, bool required) -> const float * {
        if (!okay) return nullptr;
        const std::string full = m.alias + "." + local;
        auto it = m.values.find(full);
        if (it == m.values.end()) {
            if (required) okay = fail(error, "missing SLat flow tensor: " + full);
            return nullptr;
        }
        if (it->second.size() != count) {
            okay = fail(error, "SLat flow tensor " + full + " has " + std::to_string(it->second.size()) +
                                   " values, expected " + std::to_string(count));
            return nullptr;
        }
        return it->second.data();
    };
    w.input_weight = get("input_layer.weight", C * h.in_channels, true);
    w.input_bias = get("input_layer.bias", C, true);
    w.timestep_weight0 = get("t_embedder.mlp.0.weight", C * 256, true);
    w.timestep_bias0 = get("t_embedder.mlp.0.bias", C, true);
    w.timestep_weight2 = get("t_embedder.mlp.2.weight", C * C, true);
    w.timestep_bias2 = get("t_embedder.mlp.2.bias", C, true);
    w.modulation_weight = get("adaLN_modulation.1.weight", 6 * C * C, true);
    w.modulation_bias = get("adaLN_modulation.1.bias", 6 * C, true);
    w.output_weight = get("out_layer.weight", h.out_channels * C, true);
    w.output_bias = get("out_layer.bias", h.out_channels, true);
    w.blocks.clear();
    for (int b = 0; b < h.num_blocks && okay; ++b) {
        const std::string p = "blocks." + std::to_string(b);
        const std::string cross = p + ".cross_attn.cross_attn_block";
        const std::string mp = p + ".mlp.mlp";
        SparseTransformerBlockWeightsF32 o;
        o.modulation = get(p + ".modulation", 6 * C, true);
        o.self_to_qkv_weight = get(p + ".self_attn.to_qkv.weight", 3 * C * C, true);
        o.self_to_qkv_bias = get(p + ".self_attn.to_qkv.bias", 3 * C, true);
        o.self_q_gamma = get(p + ".self_attn.q_rms_norm.gamma", C, h.qk_rms_norm);
        o.self_k_gamma = get(p + ".self_attn.k_rms_norm.gamma", C, h.qk_rms_norm);
        o.self_to_out_weight = get(p + ".self_attn.to_out.weight", C * C, true);
        o.self_to_out_bias = get(p + ".self_attn.to_out.bias", C, true);
        o.norm2_weight = get(p + ".norm2.weight", C, true);
        o.norm2_bias = get(p + ".norm2.bias", C, true);
        o.cross_to_q_weight = get(cross + ".to_q.weight", C * C, true);
        o.cross_to_q_bias = get(cross + ".to_q.bias", C, true);
        o.cross_to_kv_weight = get(cross + ".to_kv.weight", 2 * C * cc, true);
        o.cross_to_kv_bias = get(cross + ".to_kv.bias", 2 * C, true);
        o.cross_q_gamma = get(cross + ".q_rms_norm.gamma", C, h.qk_rms_norm_cross);
        o.cross_k_gamma = get(cross + ".k_rms_norm.gamma", C, h.qk_rms_norm_cross);
        o.cross_to_out_weight = get(cross + ".to_out.weight", C * C, true);
        o.cross_to_out_bias = get(cross + ".to_out.bias", C, true);
        if (h.image_attn_mode == "proj") {
            o.proj_weight = get(p + ".cross_attn.proj_linear.weight", C * pin, true);
            o.proj_bias = get(p + ".cross_attn.proj_linear.bias", C, true);
        }
        o.mlp0_weight = get(mp + ".0.weight", mlp * C, true);
        o.mlp0_bias = get(mp + ".0.bias", mlp, true);
        o.mlp2_weight = get(mp + ".2.weight", C * mlp, true);
        o.mlp2_bias = get(mp + ".2.bias", C, true);
        w.blocks.push_back(o);
    }
    return okay;
}
}  // namespace

// GGUF pack loading (SLatFlowModel::load, src/slat_flow.cpp:1239-1281, with
// the pack checks of load_pack_info, src/pack.cpp:127-176): version 3,
// architecture "pixal3d", tensor-name scheme "compact-v1", component prefix
// sh512 / sh1024 / tx1024.  F32, F16 and BF16 tensors are widened to f32 on
// the host, then uploaded as for bind() (16-bit device copies).
bool SLatFlowModel::load(const std::string &path, const std::string &component, bool load_tensors,
                         std::string *error) {
    close();
    const std::string alias = compact_prefix(component);
    if (alias.empty()) return fail(error, "unsupported SLat flow component: " + component);
    b200::GgufFile f;
    if (!f.open(path, error)) return false;
    std::string arch, scheme;
    if (!f.get_string("general.architecture", arch, true, error)) return false;
    if (arch != "pixal3d") return fail(error, "unexpected GGUF architecture: " + arch);
    if (!f.get_string("pixal3d.tensor_name_scheme", scheme, true, error)) return false;
    if (scheme != "compact-v1") return fail(error, "unsupported Pixal3D tensor name scheme: " + scheme);
    const std::string prefix = alias + ".";
    if (!f.find(prefix + "input_layer.weight"))
        return fail(error, "GGUF pack does not contain SLat flow component: " + component);
    std::unique_ptr<Impl> impl(new Impl());
    impl->hp.component = component;
    impl->alias = alias;
    if (!read_flow_hparams(f, component, impl->hp, error)) return false;
    for (const b200::GgufTensor &t : f.tensors())
        if (starts_with(t.name, prefix)) impl->pack_tensors.push_back(t.name);
    if (impl->pack_tensors.empty()) return fail(error, "SLat flow component has no tensors: " + component);
    impl->tensors = static_cast<int>(impl->pack_tensors.size());
    impl->has_data = load_tensors;
    if (load_tensors) {
        for (const std::string &name : impl->pack_tensors)
            if (!f.read_f32(*f.find(name), impl->values[name], error)) return false;
        SLatFlowWeightsF32 w;
        if (!pack_weights(*impl, w, error)) return false;
        p3d_ctx *ctx = b200::context(error);
        if (!ctx) return false;
        if (device_flow_supported(impl->hp)) {
            if (!create_flow(ctx, impl->hp, w, &impl->flow, error)) return false;
        } else {
            p3d_flow_hparams check;
            if (!to_hparams(impl->hp, check, error)) return false;
            impl->host.copy(impl->hp, w);
        }
    }
    impl_ = impl.release();
    return true;
}

bool SLatFlowModel::bind(const SLatFlowHParams &hparams, const SLatFlowWeightsF32 &weights, std::string *error) {
    close();
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    auto *impl = new Impl();
    impl->hp = hparams;
    if (device_flow_supported(hparams)) {
        if (!create_flow(ctx, hparams, weights, &impl->flow, error)) {
            delete impl;
            return false;
        }
    } else {
        p3d_flow_hparams check;
        if (!to_hparams(hparams, check, error) || static_cast<int>(weights.blocks.size()) != hparams.num_blocks) {
            delete impl;
            return error && !error->empty() ? false : fail(error, "SLat flow block count mismatch");
        }
        impl->host.copy(hparams, weights);
    }
    impl->tensors = 10 + 23 * static_cast<int>(weights.blocks.size());
    impl_ = impl;
    return true;
}

bool SLatFlowModel::is_loaded() const noexcept { return impl_ != nullptr; }
bool SLatFlowModel::has_data() const noexcept { return impl_ != nullptr && impl_->has_data; }
const SLatFlowHParams &SLatFlowModel::hparams() const noexcept {
    static const SLatFlowHParams empty;
    return impl_ ? impl_->hp : empty;
}
int SLatFlowModel::tensor_count() const noexcept { return impl_ ? impl_->tensors : 0; }
bool SLatFlowModel::has_tensor(const std::string &name) const noexcept {
    if (!impl_ || impl_->alias.empty()) return false;
    const std::string full = starts_with(name, impl_->alias + ".") ? name : impl_->alias + "." + name;
    for (const std::string &t : impl_->pack_tensors)
        if (t == full) return true;
    return false;
}

bool SLatFlowModel::forward(const SparseTensorF32 &input, const float *timesteps, std::size_t timestep_count,
                            const VarLenTensorF32 &global_context, const SparseTensorF32 *projection_context,
                            SparseTensorF32 &output, std::string *error, const SparseTensorF32 *concat_condition) {
    if (!impl_) return fail(error, "SLat flow model is not loaded");
    if (!impl_->has_data) return fail(error, "SLat flow model was loaded without tensor data");
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    if (!timesteps) return fail(error, "SLat flow timesteps are null");
    if (!check_forward_inputs(input, timestep_count, global_context, projection_context, impl_->hp, concat_condition,
                              error))
        return false;
    SparseTensorF32 joined;
    if (concat_condition && !concat_features(input, *concat_condition, joined, error)) return false;
    const SparseTensorF32 &model_input = concat_condition ? joined : input;
    if (!impl_->flow)
        return composed_forward(ctx, model_input, timesteps, global_context, projection_context, impl_->hp,
                                impl_->host.w, output, error);
    return run_forward(ctx, impl_->flow, model_input, timesteps, global_context, projection_context, impl_->hp,
                       output, error);
}

bool SLatFlowModel::sample(const SparseTensorF32 &noise, const FlowEulerSamplerConfig &sampler_config,
                           const VarLenTensorF32 &global_context, const SparseTensorF32 *projection_context,
                           FlowEulerSampleF32 &output, std::string *error, const SparseTensorF32 *concat_condition) {
    if (!impl_) return fail(error, "SLat flow model is not loaded");
    if (!impl_->has_data) return fail(error, "SLat flow model was loaded without tensor data");
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    const SLatFlowHParams &h = impl_->hp;
    if (!check_forward_inputs(noise, noise.batch_size, global_context, projection_context, h, concat_condition, error))
        return false;
    const int concat_channels = concat_condition ? concat_condition->channels : 0;
    if (sampler_config.record_trajectory || h.in_channels != h.out_channels + concat_channels || !impl_->flow) {
        // host-driven loop (trajectory recorded per step), forward on the device
        VarLenTensorF32 zeros = global_context;
        std::fill(zeros.feats.begin(), zeros.feats.end(), 0.0f);
        SparseTensorF32 zproj;
        if (projection_context) {
            zproj = *projection_context;
            std::fill(zproj.feats.begin(), zproj.feats.end(), 0.0f);
        }
        std::vector<float> ts(static_cast<std::size_t>(noise.batch_size));
        FlowVelocityFn fn = [&](const SparseTensorF32 &state, float t, bool cond, SparseTensorF32 &v,
                                std::string *e) {
            std::fill(ts.begin(), ts.end(), t);
            return forward(state, ts.data(), ts.size(), cond ? global_context : zeros,
                           projection_context ? (cond ? projection_context : &zproj) : nullptr, v, e,
                           concat_condition);
        };
        return flow_euler_sample_f32(noise, sampler_config, fn, output, error);
    }
    output = FlowEulerSampleF32{};
    Buffer x, g, coords, proj, cat;
    if (!b200::validate_sparse(ctx, noise, nullptr, &x, error) || !valid_config(sampler_config, error)) return false;
    if (concat_condition && !b200::validate_sparse(ctx, *concat_condition, nullptr, &cat, error)) return false;
    // condition items: [0, I) conditional, [I, 2I) cleared to zeros by the sampler
    const int I = noise.batch_size;
    std::vector<int64_t> coff(2 * static_cast<std::size_t>(I) + 1, 0);
    for (int b = 0; b < I; ++b) coff[b + 1] = static_cast<int64_t>(global_context.offsets[b + 1]);
    for (int b = 0; b < I; ++b) coff[I + b + 1] = coff[I] + static_cast<int64_t>(global_context.offsets[b + 1]);
    std::vector<float> cond2(global_context.feats);
    cond2.resize(global_context.feats.size() * 2, 0.0f);
    if (!b200::upload(ctx, g, cond2.data(), cond2.size() * 4, error)) return false;
    if (projection_context && !b200::validate_sparse(ctx, *projection_context, nullptr, &proj, error)) return false;
    if (!prepare(ctx, impl_->flow, noise, 2, coff, coords, error)) return false;
    p3d_sampler_config c{};
    c.steps = sampler_config.steps;
    c.sigma_min = sampler_config.sigma_min;
    c.rescale_t = sampler_config.rescale_t;
    c.guidance_strength = sampler_config.guidance_strength;
    c.guidance_rescale = sampler_config.guidance_rescale;
    c.guidance_interval_min = sampler_config.guidance_interval_min;
    c.guidance_interval_max = sampler_config.guidance_interval_max;
    c.use_graph = 1;
    if (!ok(ctx,
            p3d_flow_sample_concat(impl_->flow, x.as<float>(), g.get(), P3D_F32,
                                   projection_context ? proj.as<float>() : nullptr,
                                   concat_condition ? cat.as<float>() : nullptr, concat_channels, &c),
            error))
        return false;
    output.samples = noise;
    return b200::download(ctx, output.samples.feats.data(), x, output.samples.feats.size() * 4, error);
}

}  // namespace pixal3d
