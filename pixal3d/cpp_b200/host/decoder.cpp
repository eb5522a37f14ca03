// include/pixal3d/slat_decoder.h on the B200 kernels: whole decodes run in the
// device-resident p3d_decoder (src/slat_decoder.cpp:290-455); the single-block
// functions run the same kernel sequence (:185-288).
#include "pixal3d/slat_decoder.h"

#include <cmath>

#include "device.h"
#include "ops_internal.h"

namespace pixal3d {

using b200::Buffer;
using b200::fail;
using b200::ok;
using b200::round_up;

namespace {

bool valid_eps(float eps, std::string *error) {
    if (!(eps > 0.0f) || !std::isfinite(eps)) return fail(error, "SLat decoder norm epsilon must be finite and positive");
    return true;
}

struct Staging {
    std::vector<Buffer> bufs;
    const float *put(p3d_ctx *ctx, const float *host, std::size_t count, bool &okay, std::string *error) {
        if (!host || !okay) return nullptr;
        bufs.emplace_back();
        okay = b200::upload(ctx, bufs.back(), host, count * sizeof(float), error);
        return bufs.back().as<float>();
    }
};

bool config_ok(const SLatDecoderConfig &c, std::size_t blocks, std::string *error) {
    if (c.latent_channels <= 0 || c.out_channels <= 0 || c.model_channels.empty() ||
        c.model_channels.size() != c.num_blocks.size() || c.model_channels.size() > P3D_DECODER_MAX_LEVELS)
        return fail(error, "invalid SLat decoder configuration");
    std::size_t expected = c.model_channels.size() - 1;
    for (int k : c.num_blocks) {
        if (k < 0) return fail(error, "invalid SLat decoder block count");
        expected += static_cast<std::size_t>(k);
    }
    if (blocks != expected) return fail(error, "SLat decoder weight block count does not match configuration");
    return valid_eps(c.norm_eps, error);
}

bool create_decoder(p3d_ctx *ctx, const SLatDecoderConfig &c, const SLatDecoderWeightsF32 &w, p3d_decoder **dec,
                    std::string *error) {
    if (!config_ok(c, w.blocks.size(), error)) return false;
    if (!w.from_latent_weight || !w.output_weight) return fail(error, "missing SLat decoder tensor");
    p3d_decoder_config cfg{};
    cfg.latent_channels = c.latent_channels;
    cfg.out_channels = c.out_channels;
    cfg.levels = static_cast<int>(c.model_channels.size());
    for (int l = 0; l < cfg.levels; ++l) {
        cfg.model_channels[l] = c.model_channels[l];
        cfg.num_blocks[l] = c.num_blocks[l];
    }
    cfg.pred_subdiv = c.pred_subdiv ? 1 : 0;
    cfg.norm_eps = c.norm_eps;
    cfg.operand_dtype = b200::kOperand;
    Staging st;
    bool okay = true;
    const std::size_t C0 = c.model_channels.front(), CL = c.model_channels.back();
    p3d_decoder_weights dw{};
    dw.from_latent_w = st.put(ctx, w.from_latent_weight, C0 * c.latent_channels, okay, error);
    dw.from_latent_b = st.put(ctx, w.from_latent_bias, C0, okay, error);
    dw.output_w = st.put(ctx, w.output_weight, CL * c.out_channels, okay, error);
    dw.output_b = st.put(ctx, w.output_bias, c.out_channels, okay, error);
    std::vector<p3d_decoder_block> blocks;
    st.bufs.reserve(4 + 14 * w.blocks.size());
    for (const SLatDecoderBlockWeightsF32 &b : w.blocks) {
        p3d_decoder_block o{};
        o.kind = b.kind == SLatDecoderBlockKind::convnext ? 0 : 1;
        o.channels = b.channels;
        o.out_channels = b.out_channels;
        o.mlp_hidden = b.mlp_hidden;
        const std::size_t C = b.channels, O = b.out_channels, M = b.mlp_hidden;
        if (o.kind == 0) {
            o.norm_w = st.put(ctx, b.norm_weight, C, okay, error);
            o.norm_b = st.put(ctx, b.norm_bias, C, okay, error);
            o.conv1_w = st.put(ctx, b.conv1_weight, 27 * C * C, okay, error);
            o.conv1_b = st.put(ctx, b.conv1_bias, C, okay, error);
            o.mlp0_w = st.put(ctx, b.mlp0_weight, M * C, okay, error);
            o.mlp0_b = st.put(ctx, b.mlp0_bias, M, okay, error);
            o.mlp2_w = st.put(ctx, b.mlp2_weight, C * M, okay, error);
            o.mlp2_b = st.put(ctx, b.mlp2_bias, C, okay, error);
        } else {
            o.norm1_w = st.put(ctx, b.norm1_weight, C, okay, error);
            o.norm1_b = st.put(ctx, b.norm1_bias, C, okay, error);
            o.conv1_w = st.put(ctx, b.conv1_weight, 27 * 8 * O * C, okay, error);
            o.conv1_b = st.put(ctx, b.conv1_bias, 8 * O, okay, error);
            o.conv2_w = st.put(ctx, b.conv2_weight, 27 * O * O, okay, error);
            o.conv2_b = st.put(ctx, b.conv2_bias, O, okay, error);
            o.subdiv_w = st.put(ctx, b.to_subdiv_weight, 8 * C, okay, error);
            o.subdiv_b = st.put(ctx, b.to_subdiv_bias, 8, okay, error);
        }
        blocks.push_back(o);
    }
    if (!okay) return false;
    dw.blocks = blocks.data();
    dw.num_blocks = static_cast<int>(blocks.size());
    return ok(ctx, p3d_decoder_create(ctx, &cfg, &dw, dec), error);
}

SparseTensorF32 level_tensor(const SparseTensorF32 &input, int level, int channels) {
    SparseTensorF32 t;
    t.batch_size = input.batch_size;
    t.channels = channels;
    t.spatial_x = input.spatial_x << level;
    t.spatial_y = input.spatial_y << level;
    t.spatial_z = input.spatial_z << level;
    return t;
}

bool download_level_coords(p3d_ctx *ctx, p3d_decoder *dec, int level, std::vector<int32_t> &coords,
                           std::string *error) {
    const int64_t rows = p3d_decoder_rows(dec, level);
    Buffer b;
    if (rows < 0 || !b.allocate(ctx, sizeof(int32_t) * 4 * rows, error)) return false;
    coords.resize(static_cast<std::size_t>(rows) * 4);
    return ok(ctx, p3d_decoder_coords(dec, level, b.as<int32_t>()), error) &&
           b200::download(ctx, coords.data(), b, coords.size() * 4, error);
}

// One decode (stop_level == levels) or coordinate upsample (stop_level < levels).
bool run_decoder(p3d_ctx *ctx, p3d_decoder *dec, const SLatDecoderConfig &c, const SparseTensorF32 &input,
                 const std::vector<SparseTensorF32> *guides, int stop_level, SparseTensorF32 &output,
                 std::vector<SparseTensorF32> *predicted, std::string *error) {
    Buffer c32, x32;
    if (!b200::validate_sparse(ctx, input, &c32, &x32, error)) return false;
    if (input.channels != c.latent_channels) return fail(error, "SLat decoder latent channel count does not match input");
    const int levels = static_cast<int>(c.model_channels.size());
    if (guides && static_cast<int>(guides->size()) != levels - 1)
        return fail(error, "SLat decoder guide subdivision count does not match levels");
    std::vector<Buffer> gbufs(guides ? guides->size() : 0);
    std::vector<const float *> gptr;
    std::vector<int64_t> grows;
    if (guides && !c.pred_subdiv) {
        for (std::size_t l = 0; l < guides->size(); ++l) {
            const SparseTensorF32 &g = (*guides)[l];
            if (g.channels != 8 || g.batch_size != input.batch_size)
                return fail(error, "sparse subdivision shape or coordinates do not match input");
            if (!b200::validate_sparse(ctx, g, nullptr, &gbufs[l], error)) return false;
            gptr.push_back(gbufs[l].as<float>());
            grows.push_back(static_cast<int64_t>(g.points()));
        }
    }
    if (!ok(ctx,
            p3d_decoder_run(dec, c32.as<int32_t>(), static_cast<int64_t>(input.points()), input.batch_size,
                            input.spatial_x, input.spatial_y, input.spatial_z, x32.as<float>(),
                            gptr.empty() ? nullptr : gptr.data(), grows.empty() ? nullptr : grows.data(), stop_level),
            error))
        return false;
    if (!gptr.empty()) {  // guides must sit on the decoder's own level coordinates
        for (int l = 0; l < levels - 1; ++l) {
            std::vector<int32_t> lc;
            if (!download_level_coords(ctx, dec, l, lc, error)) return false;
            if (lc != (*guides)[l].coords)
                return fail(error, "sparse subdivision shape or coordinates do not match input");
        }
    }
    const int last = stop_level < levels ? stop_level : levels - 1;
    const int cols = stop_level < levels ? c.model_channels[stop_level] : c.out_channels;
    SparseTensorF32 out = level_tensor(input, last, cols);
    if (!download_level_coords(ctx, dec, last, out.coords, error)) return false;
    Buffer y;
    const std::size_t count = out.points() * static_cast<std::size_t>(cols);
    if (!y.allocate(ctx, count * 4, error) || !ok(ctx, p3d_decoder_output(dec, y.as<float>()), error) ||
        !b200::download_feats(ctx, y, count, out.feats, error))
        return false;
    if (predicted) {
        predicted->clear();
        if (c.pred_subdiv && stop_level == levels) {
            for (int l = 0; l + 1 < levels; ++l) {
                SparseTensorF32 p = level_tensor(input, l, 8);
                if (!download_level_coords(ctx, dec, l, p.coords, error)) return false;
                Buffer pb;
                const std::size_t pc = p.points() * 8;
                if (!pb.allocate(ctx, pc * 4, error) || !ok(ctx, p3d_decoder_subdivision(dec, l, pb.as<float>()), error) ||
                    !b200::download_feats(ctx, pb, pc, p.feats, error))
                    return false;
                predicted->push_back(std::move(p));
            }
        }
    }
    output = std::move(out);
    return true;
}

// Host weights -> 16-bit operand [rows_pad][ld] on the device.
bool weight16(p3d_ctx *ctx, const float *w, int64_t rows, int64_t cols, int64_t rows_pad, int64_t ld, Buffer &out,
              std::string *error) {
    std::vector<float> p(static_cast<std::size_t>(rows_pad * ld), 0.0f);
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t k = 0; k < cols; ++k) p[r * ld + k] = w[r * cols + k];
    return b200::upload_operand(ctx, out, p.data(), rows_pad, ld, ld, error);
}

bool bias32(p3d_ctx *ctx, const float *b, int64_t n, int64_t n_pad, Buffer &out, std::string *error) {
    std::vector<float> p(static_cast<std::size_t>(n_pad), 0.0f);
    if (b)
        for (int64_t i = 0; i < n; ++i) p[i] = b[i];
    return b200::upload(ctx, out, p.data(), p.size() * 4, error);
}

bool nbr_map(p3d_ctx *ctx, const Buffer &coords, int64_t n, Buffer &nbr, std::string *error) {
    Buffer ws;
    const std::size_t wsb = p3d_neighbor_map27_workspace(n);
    return ws.allocate(ctx, wsb, error) && nbr.allocate(ctx, sizeof(int32_t) * 27 * n, error) &&
           ok(ctx, p3d_neighbor_map27_ws(ctx, coords.as<int32_t>(), n, ws.get(), wsb, nbr.as<int32_t>()), error);
}

}  // namespace

bool sparse_convnext_block_f32(const SparseTensorF32 &input, const SLatDecoderBlockWeightsF32 &w, float norm_eps,
                               SparseTensorF32 &output, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer c32, h;
    if (!b200::validate_sparse(ctx, input, &c32, &h, error) || !valid_eps(norm_eps, error)) return false;
    if (w.kind != SLatDecoderBlockKind::convnext || w.channels != input.channels || w.out_channels != input.channels ||
        w.mlp_hidden <= 0)
        return fail(error, "invalid SLat ConvNeXt block dimensions");
    if (!w.norm_weight || !w.norm_bias || !w.conv1_weight || !w.conv1_bias || !w.mlp0_weight || !w.mlp0_bias ||
        !w.mlp2_weight || !w.mlp2_bias)
        return fail(error, "missing SLat decoder tensor");
    const int C = input.channels, M = w.mlp_hidden;
    const int64_t n = static_cast<int64_t>(input.points()), Cp64 = round_up(C, 64), Ck8 = round_up(C, 8),
                  Mp = round_up(M, 8);
    const int dt = b200::kOperand;
    Buffer nbr, wc, bc, nw, nb, w0, b0, w2, b2, op, t, ln, hid;
    if (!nbr_map(ctx, c32, n, nbr, error) || !weight16(ctx, w.conv1_weight, 27LL * C, C, 27LL * C, Cp64, wc, error) ||
        !bias32(ctx, w.conv1_bias, C, C, bc, error) || !b200::upload(ctx, nw, w.norm_weight, 4 * C, error) ||
        !b200::upload(ctx, nb, w.norm_bias, 4 * C, error) || !weight16(ctx, w.mlp0_weight, M, C, Mp, Ck8, w0, error) ||
        !bias32(ctx, w.mlp0_bias, M, Mp, b0, error) || !weight16(ctx, w.mlp2_weight, C, M, C, Mp, w2, error) ||
        !bias32(ctx, w.mlp2_bias, C, C, b2, error) || !op.allocate(ctx, 2 * n * Cp64, error) ||
        !t.allocate(ctx, 4 * n * C, error) || !ln.allocate(ctx, 2 * n * Ck8, error) ||
        !hid.allocate(ctx, 2 * n * Mp, error))
        return false;
    if (n > 0 &&
        (!ok(ctx, p3d_pack_operand(ctx, h.as<float>(), n, C, op.get(), Cp64, dt), error) ||
         !ok(ctx,
             p3d_subm_conv3d(ctx, op.get(), n, Cp64, nbr.as<int32_t>(), wc.get(), dt, bc.as<float>(), C, t.get(), C,
                             P3D_F32, P3D_EPI_NONE, nullptr, 0, nullptr, 0),
             error) ||
         !ok(ctx, p3d_layernorm_act(ctx, t.as<float>(), n, C, norm_eps, nw.as<float>(), nb.as<float>(), 0, ln.get(), Ck8, dt),
             error) ||
         !ok(ctx,
             p3d_linear(ctx, ln.get(), Ck8, w0.get(), dt, b0.as<float>(), n, Mp, Ck8, hid.get(), Mp, dt, P3D_EPI_SILU,
                        nullptr, 0, nullptr, 0),
             error) ||
         !ok(ctx,
             p3d_linear(ctx, hid.get(), Mp, w2.get(), dt, b2.as<float>(), n, C, Mp, h.get(), C, P3D_F32,
                        P3D_EPI_RESIDUAL, nullptr, 0, nullptr, 0),
             error)))
        return false;
    std::vector<float> feats;
    if (!b200::download_feats(ctx, h, static_cast<std::size_t>(n) * C, feats, error)) return false;
    b200::copy_shape(input, C, output);
    output.feats = std::move(feats);
    return true;
}

bool sparse_resblock_c2s_f32(const SparseTensorF32 &input, const SLatDecoderBlockWeightsF32 &w, float norm_eps,
                             bool pred_subdiv, const SparseTensorF32 *subdivision, SparseTensorF32 &output,
                             SparseTensorF32 *predicted_subdiv, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    Buffer c32, x32, g32;
    if (!b200::validate_sparse(ctx, input, &c32, &x32, error) || !valid_eps(norm_eps, error)) return false;
    const int C = input.channels, O = w.out_channels;
    if (w.kind != SLatDecoderBlockKind::channel_to_spatial || w.channels != C || O <= 0 || C % 8 != 0)
        return fail(error, "invalid SLat channel-to-spatial block dimensions");
    if (O % (C / 8) != 0) return fail(error, "SLat decoder skip channels are not repeatable");
    if (!w.norm1_weight || !w.norm1_bias || !w.conv1_weight || !w.conv1_bias || !w.conv2_weight || !w.conv2_bias ||
        (pred_subdiv && (!w.to_subdiv_weight || !w.to_subdiv_bias)))
        return fail(error, "missing SLat decoder tensor");
    const int64_t n = static_cast<int64_t>(input.points()), Cp64 = round_up(C, 64), Ck8 = round_up(C, 8),
                  Op64 = round_up(O, 64);
    const int dt = b200::kOperand;
    Buffer sub, hk, ws8, bs8;
    const float *mask = nullptr;
    SparseTensorF32 predicted;
    if (pred_subdiv) {
        if (!hk.allocate(ctx, 2 * n * Ck8, error) || !weight16(ctx, w.to_subdiv_weight, 8, C, 8, Ck8, ws8, error) ||
            !bias32(ctx, w.to_subdiv_bias, 8, 8, bs8, error) || !sub.allocate(ctx, 4 * n * 8, error))
            return false;
        if (n > 0 && (!ok(ctx, p3d_pack_operand(ctx, x32.as<float>(), n, C, hk.get(), Ck8, dt), error) ||
                      !ok(ctx,
                          p3d_linear(ctx, hk.get(), Ck8, ws8.get(), dt, bs8.as<float>(), n, 8, Ck8, sub.get(), 8,
                                     P3D_F32, P3D_EPI_NONE, nullptr, 0, nullptr, 0),
                          error)))
            return false;
        mask = sub.as<float>();
        predicted = input;
        predicted.channels = 8;
        if (!b200::download_feats(ctx, sub, static_cast<std::size_t>(n) * 8, predicted.feats, error)) return false;
    } else if (subdivision) {
        if (subdivision->batch_size != input.batch_size || subdivision->channels != 8 ||
            subdivision->coords != input.coords ||
            !b200::validate_sparse(ctx, *subdivision, nullptr, &g32, error))
            return fail(error, "sparse subdivision shape or coordinates do not match input");
        mask = g32.as<float>();
    }
    Buffer nbr, nw, nb, w1, b1, w2, b2, ln1, packed, scratch, nc, src_row, src_child, dm;
    if (!nbr_map(ctx, c32, n, nbr, error) || !b200::upload(ctx, nw, w.norm1_weight, 4 * C, error) ||
        !b200::upload(ctx, nb, w.norm1_bias, 4 * C, error) ||
        !weight16(ctx, w.conv1_weight, 27LL * 8 * O, C, 27LL * 8 * O, Cp64, w1, error) ||
        !bias32(ctx, w.conv1_bias, 8LL * O, 8LL * O, b1, error) ||
        !weight16(ctx, w.conv2_weight, 27LL * O, O, 27LL * O, Op64, w2, error) ||
        !bias32(ctx, w.conv2_bias, O, O, b2, error) || !ln1.allocate(ctx, 2 * n * Cp64, error) ||
        !packed.allocate(ctx, 4 * n * 8 * O, error) || !scratch.allocate(ctx, 8 * (n + 1), error) ||
        !nc.allocate(ctx, 4 * 4 * 8 * n, error) || !src_row.allocate(ctx, 4 * 8 * n, error) ||
        !src_child.allocate(ctx, 8 * n, error) || !dm.allocate(ctx, 8, error))
        return false;
    if (!ok(ctx, p3d_layernorm_act(ctx, x32.as<float>(), n, C, norm_eps, nw.as<float>(), nb.as<float>(), 1, ln1.get(), Cp64, dt),
            error) ||
        !ok(ctx,
            p3d_subm_conv3d(ctx, ln1.get(), n, Cp64, nbr.as<int32_t>(), w1.get(), dt, b1.as<float>(), 8LL * O,
                            packed.get(), 8LL * O, P3D_F32, P3D_EPI_NONE, nullptr, 0, nullptr, 0),
            error) ||
        !ok(ctx,
            p3d_c2s_topology(ctx, c32.as<int32_t>(), n, 2, mask, scratch.as<int64_t>(), nc.as<int32_t>(),
                             src_row.as<int32_t>(), src_child.as<int8_t>(), dm.as<int64_t>()),
            error))
        return false;
    int64_t m = 0;
    if (!b200::download(ctx, &m, dm, 8, error)) return false;
    Buffer hs, hn, ln2, nbr2;
    if (!hs.allocate(ctx, 4 * m * O, error) || !hn.allocate(ctx, 4 * m * O, error) ||
        !ln2.allocate(ctx, 2 * m * Op64, error))
        return false;
    if (m > 0 &&
        (!ok(ctx, p3d_c2s_gather(ctx, packed.get(), 8LL * O, src_row.as<int32_t>(), src_child.as<int8_t>(), m, O, 1, P3D_F32, hs.get()),
             error) ||
         !ok(ctx,
             p3d_c2s_gather(ctx, x32.get(), C, src_row.as<int32_t>(), src_child.as<int8_t>(), m, C / 8, O / (C / 8),
                            P3D_F32, hn.get()),
             error) ||
         !ok(ctx, p3d_layernorm_act(ctx, hs.as<float>(), m, O, norm_eps, nullptr, nullptr, 1, ln2.get(), Op64, dt), error) ||
         !nbr_map(ctx, nc, m, nbr2, error) ||
         !ok(ctx,
             p3d_subm_conv3d(ctx, ln2.get(), m, Op64, nbr2.as<int32_t>(), w2.get(), dt, b2.as<float>(), O, hn.get(), O,
                             P3D_F32, P3D_EPI_RESIDUAL, nullptr, 0, nullptr, 0),
             error)))
        return false;
    SparseTensorF32 out = level_tensor(input, 1, O);
    out.coords.resize(static_cast<std::size_t>(m) * 4);
    if (!b200::download(ctx, out.coords.data(), nc, out.coords.size() * 4, error) ||
        !b200::download_feats(ctx, hn, static_cast<std::size_t>(m) * O, out.feats, error))
        return false;
    if (predicted_subdiv) *predicted_subdiv = pred_subdiv ? std::move(predicted) : SparseTensorF32{};
    output = std::move(out);
    return true;
}

bool slat_decoder_forward_f32(const SparseTensorF32 &input, const SLatDecoderConfig &config,
                              const SLatDecoderWeightsF32 &weights,
                              const std::vector<SparseTensorF32> *guide_subdivisions, SparseTensorF32 &output,
                              std::vector<SparseTensorF32> *predicted_subdivisions, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    p3d_decoder *dec = nullptr;
    if (!create_decoder(ctx, config, weights, &dec, error)) return false;
    const bool r = run_decoder(ctx, dec, config, input, guide_subdivisions,
                               static_cast<int>(config.model_channels.size()), output, predicted_subdivisions, error);
    p3d_decoder_destroy(dec);
    return r;
}

bool slat_decoder_upsample_coords_f32(const SparseTensorF32 &input, const SLatDecoderConfig &config,
                                      const SLatDecoderWeightsF32 &weights, int upsample_times,
                                      SparseTensorF32 &output, std::string *error) {
    output = SparseTensorF32{};
    if (!config.pred_subdiv || upsample_times < 0 ||
        upsample_times >= static_cast<int>(config.model_channels.size()))
        return fail(error, "invalid SLat decoder coordinate-upsample configuration");
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    p3d_decoder *dec = nullptr;
    if (!create_decoder(ctx, config, weights, &dec, error)) return false;
    const bool r = run_decoder(ctx, dec, config, input, nullptr, upsample_times, output, nullptr, error);
    p3d_decoder_destroy(dec);
    return r;
}

struct SLatDecoderModel::Impl {
    SLatDecoderHParams hp;
    SLatDecoderConfig cfg;
    p3d_decoder *dec = nullptr;
    int tensors = 0;
    ~Impl() {
        if (dec) p3d_decoder_destroy(dec);
    }
};

SLatDecoderModel::~SLatDecoderModel() { close(); }

void SLatDecoderModel::close() noexcept {
    delete impl_;
    impl_ = nullptr;
}

bool SLatDecoderModel::load(const std::string &, const std::string &, bool, std::string *error) {
    return fail(error, "SLat decoder weight packs are not read by the B200 build; bind host weights with bind()");
}

bool SLatDecoderModel::bind(const SLatDecoderHParams &hp, const SLatDecoderWeightsF32 &weights, std::string *error) {
    close();
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    auto *impl = new Impl();
    impl->hp = hp;
    impl->cfg.latent_channels = hp.latent_channels;
    impl->cfg.out_channels = hp.out_channels;
    impl->cfg.norm_eps = hp.norm_eps;
    impl->cfg.pred_subdiv = hp.pred_subdiv;
    impl->cfg.model_channels = hp.model_channels;
    impl->cfg.num_blocks = hp.num_blocks;
    if (!create_decoder(ctx, impl->cfg, weights, &impl->dec, error)) {
        delete impl;
        return false;
    }
    impl->tensors = 4 + static_cast<int>(weights.blocks.size()) * 8;
    impl_ = impl;
    return true;
}

bool SLatDecoderModel::is_loaded() const noexcept { return impl_ != nullptr; }
bool SLatDecoderModel::has_data() const noexcept { return impl_ != nullptr; }
const SLatDecoderHParams &SLatDecoderModel::hparams() const noexcept {
    static const SLatDecoderHParams empty;
    return impl_ ? impl_->hp : empty;
}
int SLatDecoderModel::tensor_count() const noexcept { return impl_ ? impl_->tensors : 0; }
bool SLatDecoderModel::has_tensor(const std::string &) const noexcept { return false; }

bool SLatDecoderModel::decode(const SparseTensorF32 &input, const std::vector<SparseTensorF32> *guide_subdivisions,
                              SparseTensorF32 &output, std::vector<SparseTensorF32> *predicted_subdivisions,
                              std::string *error) {
    if (!impl_) return fail(error, "SLat decoder model is not loaded");
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    if (!impl_->hp.pred_subdiv &&
        (!guide_subdivisions || guide_subdivisions->size() != impl_->hp.model_channels.size() - 1))
        return fail(error, "texture SLat decoder requires one guide subdivision per upsample level");
    return run_decoder(ctx, impl_->dec, impl_->cfg, input, guide_subdivisions,
                       static_cast<int>(impl_->cfg.model_channels.size()), output, predicted_subdivisions, error);
}

bool SLatDecoderModel::upsample_coords(const SparseTensorF32 &input, int upsample_times, SparseTensorF32 &output,
                                       std::string *error) {
    if (!impl_) return fail(error, "SLat decoder model is not loaded");
    if (!impl_->hp.pred_subdiv || upsample_times < 0 ||
        upsample_times >= static_cast<int>(impl_->cfg.model_channels.size()))
        return fail(error, "invalid SLat decoder coordinate-upsample configuration");
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    return run_decoder(ctx, impl_->dec, impl_->cfg, input, nullptr, upsample_times, output, nullptr, error);
}

}  // namespace pixal3d
