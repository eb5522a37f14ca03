// sparse_transformer_cross_block_f32 on the B200 kernels: the residual
// stream stays on the device (f32) for the whole block; LayerNorm +
// AdaLN modulation feed 16-bit GEMM operands; gates and residual adds are
// GEMM epilogues (src/sparse_transformer.cpp:138-292).
#include "pixal3d/sparse_transformer.h"

#include <cmath>

#include "device.h"
#include "ops_internal.h"

namespace pixal3d {

using b200::Buffer;
using b200::fail;
using b200::ok;
using b200::round_up;

namespace {

bool need(const float *p, const char *name, std::string *error) {
    if (p) return true;
    if (error) *error = std::string("missing sparse transformer tensor: ") + name;
    return false;
}

// Host f32 [out][in] -> device 16-bit [out_pad][in_pad] (zero padded) and
// f32 bias [out_pad] (zero padded; null bias -> zeros).
struct Weight {
    Buffer w, b;
    int64_t out_pad = 0, in_pad = 0;
    bool load(p3d_ctx *ctx, const float *wh, const float *bh, int out, int in, int64_t out_pad_, int64_t in_pad_,
              std::string *error) {
        out_pad = out_pad_;
        in_pad = in_pad_;
        std::vector<float> wp(static_cast<std::size_t>(out_pad * in_pad), 0.0f);
        for (int o = 0; o < out; ++o)
            for (int i = 0; i < in; ++i) wp[o * in_pad + i] = wh[static_cast<std::size_t>(o) * in + i];
        std::vector<float> bp(static_cast<std::size_t>(out_pad), 0.0f);
        if (bh)
            for (int o = 0; o < out; ++o) bp[o] = bh[o];
        return b200::upload_operand(ctx, w, wp.data(), out_pad, in_pad, in_pad, error) &&
               b200::upload(ctx, b, bp.data(), bp.size() * sizeof(float), error);
    }
};

struct BlockRun {
    p3d_ctx *ctx;
    std::string *error;
    int64_t n, C, Cp;
    int B;
    Buffer offs, mods;  // batch offsets [B+1], per-item modulation [B][6C]

    // LayerNorm (+AdaLN shift/scale at mod_col, or affine) of h -> 16-bit [n][Cp].
    bool norm(const Buffer &h, float eps, const float *gamma_dev, const float *beta_dev, int64_t mod_col, Buffer &out) {
        const float *mod = mod_col >= 0 ? mods.as<float>() + mod_col : nullptr;
        if (Cp == C) {
            if (!out.allocate(ctx, static_cast<std::size_t>(n) * Cp * 2, error)) return false;
            return n == 0 || ok(ctx,
                                p3d_layernorm_modulate(ctx, h.as<float>(), n, static_cast<int>(C), eps, gamma_dev,
                                                       beta_dev, mod, 6 * C, offs.as<int32_t>(), B, out.get(),
                                                       b200::kOperand),
                                error);
        }
        Buffer tmp;
        if (!tmp.allocate(ctx, static_cast<std::size_t>(n) * C * 2, error) ||
            !out.allocate(ctx, static_cast<std::size_t>(n) * Cp * 2, error))
            return false;
        return n == 0 ||
               (ok(ctx,
                   p3d_layernorm_modulate(ctx, h.as<float>(), n, static_cast<int>(C), eps, gamma_dev, beta_dev, mod,
                                          6 * C, offs.as<int32_t>(), B, tmp.get(), b200::kOperand),
                   error) &&
                ok(ctx,
                   p3d_repack_heads(ctx, tmp.get(), C, n, 1, static_cast<int>(C), static_cast<int>(C), out.get(), Cp,
                                    b200::kOperand),
                   error));
    }
    // out16 [rows][W.out_pad] = x16 W^T + b (16-bit out), or residual add
    // into the f32 stream h (gated by mods[gate_col] when gate_col >= 0).
    bool gemm16(const void *x16, int64_t rows, const Weight &W, int epi, Buffer &out) {
        if (!out.allocate(ctx, static_cast<std::size_t>(rows) * W.out_pad * 2, error)) return false;
        return rows == 0 || ok(ctx,
                               p3d_linear(ctx, x16, W.in_pad, W.w.get(), b200::kOperand, W.b.as<float>(), rows,
                                          W.out_pad, W.in_pad, out.get(), W.out_pad, b200::kOperand, epi, nullptr, 0,
                                          nullptr, 0),
                               error);
    }
    bool residual(const void *x16, const Weight &W, Buffer &h, int64_t gate_col) {
        return n == 0 || ok(ctx,
                            p3d_linear(ctx, x16, W.in_pad, W.w.get(), b200::kOperand, W.b.as<float>(), n, C, W.in_pad,
                                       h.get(), C, P3D_F32, P3D_EPI_RESIDUAL,
                                       gate_col >= 0 ? mods.as<float>() + gate_col : nullptr, 6 * C,
                                       gate_col >= 0 ? offs.as<int32_t>() : nullptr, gate_col >= 0 ? B : 0),
                            error);
    }
};

}  // namespace

namespace b200 {

bool block_device(p3d_ctx *ctx, Buffer &h, const BlockInputs &in, const float *timestep_modulation,
                  const SparseTransformerBlockConfig &config, const SparseTransformerBlockWeightsF32 &weights,
                  std::string *error) {
    const int C = config.channels, H = config.num_heads, hd = C / H;
    if (hd > 64 || hd % 2 != 0)
        return fail(error, "sparse transformer head_dim must be even and at most 64 on the B200 kernels");
    const SparseTransformerBlockWeightsF32 &w = weights;
    if (!need(w.modulation, "modulation", error) || !need(w.self_to_qkv_weight, "self_attn.to_qkv.weight", error) ||
        !need(w.self_to_qkv_bias, "self_attn.to_qkv.bias", error) ||
        !need(w.self_to_out_weight, "self_attn.to_out.weight", error) ||
        !need(w.self_to_out_bias, "self_attn.to_out.bias", error) || !need(w.norm2_weight, "norm2.weight", error) ||
        !need(w.norm2_bias, "norm2.bias", error) || !need(w.cross_to_q_weight, "cross_attn.to_q.weight", error) ||
        !need(w.cross_to_q_bias, "cross_attn.to_q.bias", error) ||
        !need(w.cross_to_kv_weight, "cross_attn.to_kv.weight", error) ||
        !need(w.cross_to_kv_bias, "cross_attn.to_kv.bias", error) ||
        !need(w.cross_to_out_weight, "cross_attn.to_out.weight", error) ||
        !need(w.cross_to_out_bias, "cross_attn.to_out.bias", error) ||
        !need(w.mlp0_weight, "mlp.mlp.0.weight", error) || !need(w.mlp0_bias, "mlp.mlp.0.bias", error) ||
        !need(w.mlp2_weight, "mlp.mlp.2.weight", error) || !need(w.mlp2_bias, "mlp.mlp.2.bias", error))
        return false;
    if (config.qk_rms_norm && (!need(w.self_q_gamma, "self_attn.q_rms_norm.gamma", error) ||
                               !need(w.self_k_gamma, "self_attn.k_rms_norm.gamma", error)))
        return false;
    if (config.qk_rms_norm_cross && (!need(w.cross_q_gamma, "cross_attn.q_rms_norm.gamma", error) ||
                                     !need(w.cross_k_gamma, "cross_attn.k_rms_norm.gamma", error)))
        return false;
    if (config.use_projection && (!need(w.proj_weight, "cross_attn.proj_linear.weight", error) ||
                                  !need(w.proj_bias, "cross_attn.proj_linear.bias", error)))
        return false;

    BlockRun r{ctx, error, in.n, C, round_up(C, 8), in.batch, {}, {}};
    const int64_t n = r.n, Cp = r.Cp, T = static_cast<int64_t>(in.ctx_offsets.back());
    const std::vector<int32_t> &fine = in.offsets, &coff = in.ctx_offsets;
    std::vector<float> mods(static_cast<std::size_t>(r.B) * 6 * C);
    for (int b = 0; b < r.B; ++b)
        for (int j = 0; j < 6 * C; ++j)
            mods[static_cast<std::size_t>(b) * 6 * C + j] =
                w.modulation[j] + timestep_modulation[static_cast<std::size_t>(b) * 6 * C + j];
    if (!b200::upload(ctx, r.offs, fine.data(), fine.size() * 4, error) ||
        !b200::upload(ctx, r.mods, mods.data(), mods.size() * 4, error))
        return false;
    for (int b = 0; b < r.B; ++b)
        if (fine[b + 1] > fine[b] && coff[b + 1] == coff[b])
            return fail(error, "sparse cross-attention has an empty key sequence");

    // weights (16-bit, padded); qkv rows padded so q, k, v each start on an 8-column boundary
    const int64_t Cq = round_up(C, 8), mlp_p = round_up(config.mlp_hidden, 8);
    const int64_t ctxp = round_up(config.context_channels, 8);
    Weight wqkv, wout, wcq, wkv, wco, wproj, wm0, wm2;
    {
        std::vector<float> qkv_w(static_cast<std::size_t>(3 * Cq) * C, 0.0f), qkv_b(static_cast<std::size_t>(3 * Cq), 0.0f);
        for (int part = 0; part < 3; ++part)
            for (int o = 0; o < C; ++o) {
                for (int i = 0; i < C; ++i)
                    qkv_w[(part * Cq + o) * C + i] = w.self_to_qkv_weight[static_cast<std::size_t>(part * C + o) * C + i];
                qkv_b[part * Cq + o] = w.self_to_qkv_bias[part * C + o];
            }
        std::vector<float> kv_w(static_cast<std::size_t>(2 * Cq) * config.context_channels, 0.0f),
            kv_b(static_cast<std::size_t>(2 * Cq), 0.0f);
        for (int part = 0; part < 2; ++part)
            for (int o = 0; o < C; ++o) {
                for (int i = 0; i < config.context_channels; ++i)
                    kv_w[(part * Cq + o) * config.context_channels + i] =
                        w.cross_to_kv_weight[static_cast<std::size_t>(part * C + o) * config.context_channels + i];
                kv_b[part * Cq + o] = w.cross_to_kv_bias[part * C + o];
            }
        if (!wqkv.load(ctx, qkv_w.data(), qkv_b.data(), static_cast<int>(3 * Cq), C, 3 * Cq, Cp, error) ||
            !wout.load(ctx, w.self_to_out_weight, w.self_to_out_bias, C, C, C, Cp, error) ||
            !wcq.load(ctx, w.cross_to_q_weight, w.cross_to_q_bias, C, C, Cq, Cp, error) ||
            !wkv.load(ctx, kv_w.data(), kv_b.data(), static_cast<int>(2 * Cq), config.context_channels, 2 * Cq, ctxp,
                      error) ||
            !wco.load(ctx, w.cross_to_out_weight, w.cross_to_out_bias, C, C, C, Cp, error) ||
            !wm0.load(ctx, w.mlp0_weight, w.mlp0_bias, config.mlp_hidden, C, mlp_p, Cp, error) ||
            !wm2.load(ctx, w.mlp2_weight, w.mlp2_bias, C, config.mlp_hidden, C, mlp_p, error))
            return false;
        if (config.use_projection &&
            !wproj.load(ctx, w.proj_weight, w.proj_bias, C, config.proj_in_channels, C,
                        round_up(config.proj_in_channels, 8), error))
            return false;
    }
    Buffer qg, kg, cqg, ckg, n2w, n2b;
    if ((config.qk_rms_norm && (!b200::upload(ctx, qg, w.self_q_gamma, 4 * C, error) ||
                                !b200::upload(ctx, kg, w.self_k_gamma, 4 * C, error))) ||
        (config.qk_rms_norm_cross && (!b200::upload(ctx, cqg, w.cross_q_gamma, 4 * C, error) ||
                                      !b200::upload(ctx, ckg, w.cross_k_gamma, 4 * C, error))) ||
        !b200::upload(ctx, n2w, w.norm2_weight, 4 * C, error) || !b200::upload(ctx, n2b, w.norm2_bias, 4 * C, error))
        return false;

    const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
    const int dt = b200::kOperand;
    // ---- self-attention (src/sparse_transformer.cpp:194-235)
    Buffer xn, qkv, att;
    if (!r.norm(h, config.norm_eps, nullptr, nullptr, 0, xn) || !r.gemm16(xn.get(), n, wqkv, P3D_EPI_NONE, qkv))
        return false;
    uint16_t *q = qkv.as<uint16_t>(), *k = q + Cq, *v = q + 2 * Cq;
    const int32_t *rope = config.use_rope ? in.coords->as<int32_t>() : nullptr;
    if (n > 0 && (config.qk_rms_norm || rope) &&
        (!ok(ctx,
             p3d_qk_rmsnorm_rope(ctx, q, n, 3 * Cq, H, hd, config.qk_rms_norm ? qg.as<float>() : nullptr, rope,
                                 config.rope_freq_min, config.rope_freq_base, dt),
             error) ||
         !ok(ctx,
             p3d_qk_rmsnorm_rope(ctx, k, n, 3 * Cq, H, hd, config.qk_rms_norm ? kg.as<float>() : nullptr, rope,
                                 config.rope_freq_min, config.rope_freq_base, dt),
             error)))
        return false;
    if (!b200::attention16(ctx, q, 3 * Cq, n, k, 3 * Cq, v, 3 * Cq, n, fine, fine, H, hd, scale, att, Cp, error) ||
        !r.residual(att.get(), wout, h, 2 * C))
        return false;
    // ---- cross-attention (:237-275)
    Buffer xn2, cq, ctx16, kv, catt;
    if (!r.norm(h, config.norm_eps, n2w.as<float>(), n2b.as<float>(), -1, xn2) ||
        !r.gemm16(xn2.get(), n, wcq, P3D_EPI_NONE, cq) ||
        !b200::to_operand(ctx, *in.ctx32, in.ctx_host, T, config.context_channels, ctxp, ctx16, error) ||
        !r.gemm16(ctx16.get(), T, wkv, P3D_EPI_NONE, kv))
        return false;
    if (config.qk_rms_norm_cross &&
        ((n > 0 && !ok(ctx, p3d_qk_rmsnorm_rope(ctx, cq.get(), n, Cq, H, hd, cqg.as<float>(), nullptr, 1.0f, 10000.0f, dt),
                       error)) ||
         (T > 0 && !ok(ctx,
                       p3d_qk_rmsnorm_rope(ctx, kv.get(), T, 2 * Cq, H, hd, ckg.as<float>(), nullptr, 1.0f, 10000.0f,
                                           dt),
                       error))))
        return false;
    uint16_t *kc = kv.as<uint16_t>(), *vc = kc + Cq;
    if (!b200::attention16(ctx, cq.get(), Cq, n, kc, 2 * Cq, vc, 2 * Cq, T, fine, coff, H, hd, scale, catt, Cp,
                           error) ||
        !r.residual(catt.get(), wco, h, -1))
        return false;
    if (config.use_projection) {
        Buffer p16;
        const int64_t pp = round_up(config.proj_in_channels, 8);
        if (!b200::to_operand(ctx, *in.proj32, in.proj_host, n, config.proj_in_channels, pp, p16, error) ||
            !r.residual(p16.get(), wproj, h, -1))
            return false;
    }
    // ---- MLP (:277-290)
    Buffer xn3, hid;
    if (!r.norm(h, config.norm_eps, nullptr, nullptr, 3 * C, xn3) ||
        !r.gemm16(xn3.get(), n, wm0, P3D_EPI_GELU_TANH, hid) || !r.residual(hid.get(), wm2, h, 5 * C))
        return false;
    return true;
}

}  // namespace b200

bool sparse_transformer_cross_block_f32(const SparseTensorF32 &input, const float *timestep_modulation,
                                        const VarLenTensorF32 &global_context,
                                        const SparseTensorF32 *projected_context,
                                        const SparseTransformerBlockConfig &config,
                                        const SparseTransformerBlockWeightsF32 &weights, SparseTensorF32 &output,
                                        std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer c32, h, ctx32, proj32;
    if (!b200::validate_sparse(ctx, input, &c32, &h, error) ||
        !b200::validate_varlen(ctx, global_context, &ctx32, error))
        return false;
    if (!timestep_modulation || config.channels <= 0 || config.num_heads <= 0 || config.mlp_hidden <= 0 ||
        config.context_channels <= 0 || config.channels % config.num_heads != 0 ||
        input.channels != config.channels || global_context.channels != config.context_channels ||
        global_context.batch_size != input.batch_size || !(config.norm_eps > 0.0f) || !std::isfinite(config.norm_eps))
        return fail(error, "invalid sparse transformer block configuration");
    if (config.use_projection) {
        if (config.proj_in_channels <= 0 || !projected_context ||
            projected_context->channels != config.proj_in_channels ||
            projected_context->batch_size != input.batch_size || projected_context->coords != input.coords)
            return fail(error, "sparse transformer projection shape does not match query");
        if (!b200::validate_sparse(ctx, *projected_context, nullptr, &proj32, error)) return false;
    }
    b200::BlockInputs in{&c32, b200::batch_offsets(input), input.batch_size, static_cast<int64_t>(input.points()),
                         &ctx32, global_context.feats.data(), b200::varlen_offsets(global_context),
                         config.use_projection ? &proj32 : nullptr,
                         config.use_projection ? projected_context->feats.data() : nullptr};
    if (!b200::block_device(ctx, h, in, timestep_modulation, config, weights, error)) return false;
    std::vector<float> feats;
    if (!b200::download_feats(ctx, h, input.points() * static_cast<std::size_t>(config.channels), feats, error))
        return false;
    b200::copy_shape(input, config.channels, output);
    output.feats = std::move(feats);
    return true;
}

}  // namespace pixal3d
