// Runs the reference's numeric fixtures through the B200 build of the
// reference C++ API (include/pixal3d/*.h kept as declared there): the same
// calls the reference's tests/*_numeric_fixture.cpp make, on inputs read
// from a file, results written to a file for the Python test to compare
// with the reference's own outputs.
//
//   host_api_check <inputs.bin> <outputs.bin> [<flow pack.gguf> [<texture pack.gguf>]]
//
// File format: records of {u32 name length, name, u8 type (0 f32, 1 i32,
// 2 i64), u64 count, count values}.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <map>
#include <string>
#include <vector>

#include "pixal3d/flow_sampler.h"
#include "pixal3d/pipeline.h"
#include "pixal3d/slat_decoder.h"
#include "pixal3d/slat_flow.h"
#include "pixal3d/sparse.h"
#include "pixal3d/sparse_transformer.h"

using namespace pixal3d;

namespace {

struct Arr {
    uint8_t type = 0;
    std::vector<float> f;
    std::vector<int32_t> i;
    std::vector<int64_t> l;
};
std::map<std::string, Arr> in;
std::ofstream out_file;
int failures = 0;

bool read_inputs(const char *path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    while (true) {
        uint32_t len = 0;
        if (!f.read(reinterpret_cast<char *>(&len), 4)) break;
        std::string name(len, '\0');
        f.read(&name[0], len);
        Arr a;
        uint64_t count = 0;
        f.read(reinterpret_cast<char *>(&a.type), 1);
        f.read(reinterpret_cast<char *>(&count), 8);
        if (a.type == 0) {
            a.f.resize(count);
            f.read(reinterpret_cast<char *>(a.f.data()), count * 4);
        } else if (a.type == 1) {
            a.i.resize(count);
            f.read(reinterpret_cast<char *>(a.i.data()), count * 4);
        } else {
            a.l.resize(count);
            f.read(reinterpret_cast<char *>(a.l.data()), count * 8);
        }
        in[name] = std::move(a);
    }
    return true;
}

void put(const std::string &name, const std::vector<float> &v) {
    const uint32_t len = static_cast<uint32_t>(name.size());
    const uint8_t type = 0;
    const uint64_t count = v.size();
    out_file.write(reinterpret_cast<const char *>(&len), 4);
    out_file.write(name.data(), len);
    out_file.write(reinterpret_cast<const char *>(&type), 1);
    out_file.write(reinterpret_cast<const char *>(&count), 8);
    out_file.write(reinterpret_cast<const char *>(v.data()), count * 4);
}
void put(const std::string &name, const std::vector<int32_t> &v) {
    std::vector<float> f(v.begin(), v.end());
    put(name, f);
}
void put_error(const std::string &name, const std::string &err) {
    std::cerr << name << ": " << err << "\n";
    ++failures;
}

const std::vector<float> &F(const std::string &n) { return in.at(n).f; }
const std::vector<int32_t> &I(const std::string &n) { return in.at(n).i; }

SparseTensorF32 sparse(const std::vector<int32_t> &coords, const std::vector<float> &feats, int channels, int batch,
                       int sx, int sy, int sz) {
    SparseTensorF32 t;
    t.batch_size = batch;
    t.channels = channels;
    t.spatial_x = sx;
    t.spatial_y = sy;
    t.spatial_z = sz;
    t.coords = coords;
    t.feats = feats;
    return t;
}

VarLenTensorF32 varlen(const std::vector<float> &feats, int channels, const std::vector<std::size_t> &offs) {
    VarLenTensorF32 t;
    t.batch_size = static_cast<int>(offs.size()) - 1;
    t.channels = channels;
    t.offsets = offs;
    t.feats = feats;
    return t;
}

SparseTransformerBlockWeightsF32 block_weights(const std::string &p) {
    SparseTransformerBlockWeightsF32 w;
    auto g = [&](const char *n) { return F(p + n).data(); };
    w.modulation = g("modulation");
    w.self_to_qkv_weight = g("self_to_qkv_weight");
    w.self_to_qkv_bias = g("self_to_qkv_bias");
    w.self_q_gamma = g("self_q_gamma");
    w.self_k_gamma = g("self_k_gamma");
    w.self_to_out_weight = g("self_to_out_weight");
    w.self_to_out_bias = g("self_to_out_bias");
    w.norm2_weight = g("norm2_weight");
    w.norm2_bias = g("norm2_bias");
    w.cross_to_q_weight = g("cross_to_q_weight");
    w.cross_to_q_bias = g("cross_to_q_bias");
    w.cross_to_kv_weight = g("cross_to_kv_weight");
    w.cross_to_kv_bias = g("cross_to_kv_bias");
    w.cross_q_gamma = g("cross_q_gamma");
    w.cross_k_gamma = g("cross_k_gamma");
    w.cross_to_out_weight = g("cross_to_out_weight");
    w.cross_to_out_bias = g("cross_to_out_bias");
    w.proj_weight = g("proj_weight");
    w.proj_bias = g("proj_bias");
    w.mlp0_weight = g("mlp0_weight");
    w.mlp0_bias = g("mlp0_bias");
    w.mlp2_weight = g("mlp2_weight");
    w.mlp2_bias = g("mlp2_bias");
    return w;
}

void sparse_ops() {
    const SparseTensorF32 x = sparse(I("sp.coords"), F("sp.x"), 3, 2, 4, 4, 4);
    std::string e;
    SparseTensorF32 o;
    if (sparse_linear(x, F("sp.lin_w").data(), F("sp.lin_b").data(), 4, o, &e)) put("sparse_linear_output", o.feats);
    else put_error("sparse_linear", e);
    if (sparse_submanifold_conv3d(x, F("sp.conv_w").data(), F("sp.conv_b").data(), 4, o, &e))
        put("sparse_conv_output", o.feats);
    else put_error("sparse_conv", e);
    if (sparse_layer_norm(x, 1e-5f, F("sp.gamma").data(), F("sp.beta").data(), o, &e)) put("sparse_norm_output", o.feats);
    else put_error("sparse_norm", e);
    if (sparse_downsample_mean(x, 2, o, &e)) {
        put("sparse_downsample_coords", o.coords);
        put("sparse_downsample_output", o.feats);
    } else put_error("sparse_downsample", e);
    const SparseTensorF32 q = sparse(I("sp.coords"), F("sp.q"), 12, 2, 4, 4, 4);
    const SparseTensorF32 k = sparse(I("sp.coords"), F("sp.k"), 12, 2, 4, 4, 4);
    const SparseTensorF32 v = sparse(I("sp.coords"), F("sp.v"), 12, 2, 4, 4, 4);
    if (sparse_scaled_dot_product_attention(q, k, v, 2, 6, 0.37f, o, &e)) put("sparse_attention_output", o.feats);
    else put_error("sparse_attention", e);
    if (sparse_rotary_position_embedding(q, 2, 6, 1.0f, 10000.0f, o, &e)) put("sparse_rope_output", o.feats);
    else put_error("sparse_rope", e);
    if (sparse_multihead_rms_norm(q, 2, 6, F("sp.rms_gamma").data(), o, &e)) put("sparse_rms_output", o.feats);
    else put_error("sparse_rms", e);
    const VarLenTensorF32 ck = varlen(F("sp.ctx_k"), 12, {0, 3, 5}), cv = varlen(F("sp.ctx_v"), 12, {0, 3, 5});
    if (sparse_cross_attention(q, ck, cv, 2, 6, 0.29f, o, &e)) put("sparse_cross_output", o.feats);
    else put_error("sparse_cross", e);
    const SparseTensorF32 packed = sparse(I("sp.packed_coords"), F("sp.packed"), 16, 2, 2, 2, 2);
    const SparseTensorF32 sub = sparse(I("sp.packed_coords"), F("sp.subdiv"), 8, 2, 2, 2, 2);
    if (sparse_channel_to_spatial(packed, 2, &sub, o, &e)) {
        put("sparse_channel_to_spatial_coords", o.coords);
        put("sparse_channel_to_spatial_output", o.feats);
    } else put_error("sparse_channel_to_spatial", e);
    // invalid inputs report the reference's messages
    SparseTensorF32 bad = x;
    bad.coords[5 * 4 + 1] = 7;
    if (sparse_linear(bad, F("sp.lin_w").data(), F("sp.lin_b").data(), 4, o, &e) ||
        e != "sparse coordinate is outside its shape")
        put_error("invalid_outside", "expected the outside-shape error, got: " + e);
    bad = x;
    bad.coords[6 * 4 + 0] = 0;
    for (int a = 1; a < 4; ++a) bad.coords[6 * 4 + a] = x.coords[1 * 4 + a];
    if (sparse_layer_norm(bad, 1e-5f, nullptr, nullptr, o, &e) || e != "sparse coordinates contain a duplicate point")
        put_error("invalid_duplicate", "expected the duplicate error, got: " + e);
}

void block() {
    const SparseTensorF32 x = sparse(I("sp.coords"), F("blk.x"), 12, 2, 4, 4, 4);
    const SparseTensorF32 proj = sparse(I("sp.coords"), F("blk.proj"), 7, 2, 4, 4, 4);
    const VarLenTensorF32 ctx = varlen(F("blk.ctx"), 5, {0, 3, 5});
    SparseTransformerBlockConfig cfg;
    cfg.channels = 12;
    cfg.num_heads = 2;
    cfg.mlp_hidden = 18;
    cfg.context_channels = 5;
    cfg.proj_in_channels = 7;
    cfg.use_projection = true;
    SparseTensorF32 o;
    std::string e;
    if (sparse_transformer_cross_block_f32(x, F("blk.tmod").data(), ctx, &proj, cfg, block_weights("blk.w."), o, &e))
        put("sparse_transformer_output", o.feats);
    else put_error("sparse_transformer", e);
}

SLatFlowHParams flow_hp() {
    SLatFlowHParams h;
    h.in_channels = 12;
    h.out_channels = 12;
    h.model_channels = 12;
    h.cond_channels = 5;
    h.num_blocks = 1;
    h.num_heads = 2;
    h.proj_in_channels = 7;
    h.mlp_ratio = 1.5f;
    h.image_attn_mode = "proj";
    h.qk_rms_norm = true;
    h.qk_rms_norm_cross = true;
    return h;
}

void flow() {
    SLatFlowWeightsF32 w;
    w.input_weight = F("fl.input_weight").data();
    w.input_bias = F("fl.input_bias").data();
    w.timestep_weight0 = F("fl.timestep_weight0").data();
    w.timestep_bias0 = F("fl.timestep_bias0").data();
    w.timestep_weight2 = F("fl.timestep_weight2").data();
    w.timestep_bias2 = F("fl.timestep_bias2").data();
    w.modulation_weight = F("fl.modulation_weight").data();
    w.modulation_bias = F("fl.modulation_bias").data();
    w.output_weight = F("fl.output_weight").data();
    w.output_bias = F("fl.output_bias").data();
    w.blocks.push_back(block_weights("fl.b0."));
    const SparseTensorF32 x = sparse(I("sp.coords"), F("fl.x"), 12, 2, 4, 4, 4);
    const SparseTensorF32 proj = sparse(I("sp.coords"), F("fl.proj"), 7, 2, 4, 4, 4);
    const VarLenTensorF32 ctx = varlen(F("fl.ctx"), 5, {0, 3, 5});
    const SLatFlowHParams h = flow_hp();
    SparseTensorF32 o;
    std::string e;
    if (slat_flow_forward_f32(x, F("fl.timesteps").data(), 2, ctx, &proj, h, w, o, &e)) {
        put("slat_flow_coords", o.coords);
        put("slat_flow_output", o.feats);
    } else put_error("slat_flow_forward", e);
    SLatFlowModel model;
    if (!model.bind(h, w, &e)) {
        put_error("slat_flow_bind", e);
        return;
    }
    FlowEulerSamplerConfig sc;
    sc.steps = 4;
    sc.sigma_min = 0.031f;
    sc.rescale_t = 2.7f;
    sc.guidance_strength = 2.0f;
    sc.guidance_rescale = 0.23f;
    sc.guidance_interval_min = 0.34f;
    sc.guidance_interval_max = 0.91f;
    sc.record_trajectory = true;
    FlowEulerSampleF32 r;
    if (model.sample(x, sc, ctx, &proj, r, &e)) {
        put("slat_flow_sample_direct", r.samples.feats);
        put("slat_flow_sample_direct_x0_last", r.pred_x_0.back().feats);
    } else put_error("slat_flow_sample_trajectory", e);
    sc.record_trajectory = false;  // the device-resident sampler (CFG batched, one graph per step)
    if (model.sample(x, sc, ctx, &proj, r, &e)) put("slat_flow_sample_device", r.samples.feats);
    else put_error("slat_flow_sample_device", e);
    if (!model.forward(x, F("fl.timesteps").data(), 2, ctx, &proj, o, &e)) put_error("slat_flow_model_forward", e);
    else put("slat_flow_model_forward", o.feats);
}

// A model shape served by the device-resident flow (64-wide heads): forward
// and the batched-CFG device sampler through SLatFlowModel.
void flow_device() {
    if (!in.count("bf.input_weight")) return;
    SLatFlowWeightsF32 w;
    w.input_weight = F("bf.input_weight").data();
    w.input_bias = F("bf.input_bias").data();
    w.timestep_weight0 = F("bf.timestep_weight0").data();
    w.timestep_bias0 = F("bf.timestep_bias0").data();
    w.timestep_weight2 = F("bf.timestep_weight2").data();
    w.timestep_bias2 = F("bf.timestep_bias2").data();
    w.modulation_weight = F("bf.modulation_weight").data();
    w.modulation_bias = F("bf.modulation_bias").data();
    w.output_weight = F("bf.output_weight").data();
    w.output_bias = F("bf.output_bias").data();
    for (int b = 0; in.count("bf.b" + std::to_string(b) + ".modulation"); ++b)
        w.blocks.push_back(block_weights("bf.b" + std::to_string(b) + "."));
    const std::vector<float> &hpv = F("bf.hparams");  // in, out, C, cond, heads, mlp_ratio, res
    SLatFlowHParams h;
    h.in_channels = static_cast<int>(hpv[0]);
    h.out_channels = static_cast<int>(hpv[1]);
    h.model_channels = static_cast<int>(hpv[2]);
    h.cond_channels = static_cast<int>(hpv[3]);
    h.num_heads = static_cast<int>(hpv[4]);
    h.mlp_ratio = hpv[5];
    h.num_blocks = static_cast<int>(w.blocks.size());
    h.qk_rms_norm = true;
    h.qk_rms_norm_cross = true;
    const int res = static_cast<int>(hpv[6]);
    const int T = static_cast<int>(F("bf.ctx").size()) / h.cond_channels;
    const SparseTensorF32 x = sparse(I("bf.coords"), F("bf.noise"), h.in_channels, 1, res, res, res);
    const VarLenTensorF32 ctx = varlen(F("bf.ctx"), h.cond_channels, {0, static_cast<std::size_t>(T)});
    SLatFlowModel model;
    std::string e;
    if (!model.bind(h, w, &e)) {
        put_error("device_flow_bind", e);
        return;
    }
    SparseTensorF32 o;
    const float t = F("bf.timestep")[0];
    if (model.forward(x, &t, 1, ctx, nullptr, o, &e)) put("device_flow_forward", o.feats);
    else put_error("device_flow_forward", e);
    FlowEulerSamplerConfig sc;
    sc.steps = 4;
    sc.guidance_strength = 3.0f;
    sc.rescale_t = 3.0f;
    FlowEulerSampleF32 r;
    if (model.sample(x, sc, ctx, nullptr, r, &e)) put("device_flow_sample", r.samples.feats);
    else put_error("device_flow_sample", e);
}

// SLatFlowModel::load from a GGUF pack (written by tests/gguf_pack.py with
// the bf.* model's weights): header-only load, a missing component, then
// the full load and one forward on the bf.* inputs.
void flow_gguf(const std::string &path) {
    std::string e;
    {
        SLatFlowModel info;
        if (info.load(path, "shape_flow_512", false, &e)) {
            const SLatFlowHParams &h = info.hparams();
            put("gguf_info", std::vector<float>{static_cast<float>(info.tensor_count()), info.has_data() ? 1.f : 0.f,
                                                info.has_tensor("input_layer.weight") ? 1.f : 0.f,
                                                info.has_tensor("sh512.blocks.0.modulation") ? 1.f : 0.f,
                                                info.has_tensor("no.such.tensor") ? 1.f : 0.f,
                                                static_cast<float>(h.model_channels), static_cast<float>(h.num_blocks),
                                                static_cast<float>(h.num_heads), static_cast<float>(h.cond_channels),
                                                h.mlp_ratio, static_cast<float>(h.resolution)});
        } else put_error("gguf_info", e);
        SparseTensorF32 o;
        const float t = 0.5f;
        const bool fwd = info.forward(sparse(I("bf.coords"), F("bf.noise"), 8, 1, 16, 16, 16), &t, 1,
                                      varlen(F("bf.ctx"), 64, {0, F("bf.ctx").size() / 64}), nullptr, o, &e);
        put("gguf_no_data_forward_refused", std::vector<float>{fwd ? 0.f : 1.f});
    }
    {
        SLatFlowModel missing;
        const bool ok = missing.load(path, "texture_flow_1024", true, &e);
        put("gguf_missing_component_refused",
            std::vector<float>{!ok && e.find("does not contain") != std::string::npos ? 1.f : 0.f});
    }
    SLatFlowModel model;
    if (!model.load(path, "shape_flow_512", true, &e)) {
        put_error("gguf_load", e);
        return;
    }
    const SLatFlowHParams &h = model.hparams();
    const int T = static_cast<int>(F("bf.ctx").size()) / h.cond_channels;
    const SparseTensorF32 x = sparse(I("bf.coords"), F("bf.noise"), h.in_channels, 1, 16, 16, 16);
    const VarLenTensorF32 ctx = varlen(F("bf.ctx"), h.cond_channels, {0, static_cast<std::size_t>(T)});
    SparseTensorF32 o;
    const float t = F("bf.timestep")[0];
    if (model.forward(x, &t, 1, ctx, nullptr, o, &e)) put("gguf_flow_forward", o.feats);
    else put_error("gguf_flow_forward", e);
}

// The calls of the reference's tests/slat_flow_concat_fixture.cpp: a
// texture_flow_1024 pack, forward and a 3-step sample with a concat
// condition and projection context.
void flow_concat_gguf(const std::string &path) {
    std::string e;
    SLatFlowModel model;
    if (!model.load(path, "texture_flow_1024", true, &e)) {
        put_error("tx_load", e);
        return;
    }
    const SLatFlowHParams &h = model.hparams();
    const int base = 12, cc = h.in_channels - base;
    const SparseTensorF32 x = sparse(I("tx.coords"), F("tx.x"), base, 2, h.resolution, h.resolution, h.resolution);
    const SparseTensorF32 cat = sparse(I("tx.coords"), F("tx.concat"), cc, 2, h.resolution, h.resolution, h.resolution);
    const SparseTensorF32 proj =
        sparse(I("tx.coords"), F("tx.proj"), h.proj_in_channels, 2, h.resolution, h.resolution, h.resolution);
    const VarLenTensorF32 ctx = varlen(F("tx.ctx"), h.cond_channels, {0, 3, 5});
    const std::vector<float> ts = {0.17f, -0.23f};
    SparseTensorF32 o;
    if (model.forward(x, ts.data(), ts.size(), ctx, &proj, o, &e, &cat)) put("tx_concat_forward", o.feats);
    else put_error("tx_concat_forward", e);
    FlowEulerSamplerConfig sc;
    sc.steps = 3;
    sc.sigma_min = 0.031f;
    sc.rescale_t = 2.7f;
    sc.guidance_strength = 1.0f;
    sc.record_trajectory = false;
    FlowEulerSampleF32 r;
    if (model.sample(x, sc, ctx, &proj, r, &e, &cat)) put("tx_concat_sample", r.samples.feats);
    else put_error("tx_concat_sample", e);
    // the stage wrapper: sample + latent denormalization (run_slat_stage_f32)
    SLatNormalizationF32 norm;
    for (int c = 0; c < h.out_channels; ++c) {
        norm.mean.push_back(0.25f * static_cast<float>(c) - 1.0f);
        norm.std.push_back(0.5f + 0.125f * static_cast<float>(c));
    }
    Pixal3DImageConditionF32 cond{ctx, proj};
    SLatStageOutputF32 stage;
    if (run_slat_stage_f32(model, x, cond, sc, norm, stage, &e, &cat)) put("tx_stage_latent", stage.latent.feats);
    else put_error("tx_stage_latent", e);
    // a concat condition on other coordinates is refused with the reference's message
    SparseTensorF32 moved = cat;
    moved.coords[1] += 1;
    const bool refused = !model.forward(x, ts.data(), ts.size(), ctx, &proj, o, &e, &moved) &&
                         e == "SLat flow concat condition shape or coordinates mismatch";
    put("tx_concat_mismatch_refused", std::vector<float>{refused ? 1.f : 0.f});
}

// The checks of the reference's tests/pipeline_utils_test.cpp: 1 = as the
// reference asserts, 0 = not.
void pipeline_utils() {
    SparseTensorF32 up;
    up.batch_size = 1;
    up.channels = 2;
    up.spatial_x = up.spatial_y = up.spatial_z = 512;
    up.coords = {0, 0, 0, 0, 0, 1, 1, 1, 0, 256, 256, 256, 0, 511, 511, 511};
    up.feats.assign(up.points() * 2, 0.0f);
    std::vector<std::int32_t> coords;
    int res = 0;
    std::string e;
    const bool q = quantize_slat_coords_f32(up, 512, 1024, 0, coords, res, &e);
    const std::vector<std::int32_t> expected = {0, 0, 0, 0, 0, 32, 32, 32, 0, 63, 63, 63};
    std::vector<float> r = {q && res == 1024 && coords == expected ? 1.f : 0.f};
    e.clear();
    r.push_back(!quantize_slat_coords_f32(up, 512, 1536, 0, coords, res, &e) && !e.empty() ? 1.f : 0.f);
    e.clear();
    r.push_back(!quantize_slat_coords_f32(up, 512, 1024, 2, coords, res, &e) && !e.empty() ? 1.f : 0.f);
    e.clear();
    r.push_back(!quantize_slat_coords_f32(up, 512, 1000, 0, coords, res, &e) && !e.empty() ? 1.f : 0.f);
    SparseTensorF32 d;
    d.batch_size = 1;
    d.channels = 2;
    d.spatial_x = d.spatial_y = d.spatial_z = 2;
    d.coords = {0, 0, 0, 0, 0, 1, 1, 1};
    d.feats = {3.0f, -1.0f, 7.0f, 5.0f};
    SLatNormalizationF32 n;
    n.mean = {1.0f, 2.0f};
    n.std = {2.0f, 3.0f};
    SparseTensorF32 o;
    const bool nz = normalize_slat_f32(d, n, o, &e);
    const std::vector<float> en = {1.0f, -1.0f, 3.0f, 1.0f};
    bool close = nz && o.coords == d.coords && o.feats.size() == en.size();
    for (std::size_t i = 0; close && i < en.size(); ++i) close = std::fabs(o.feats[i] - en[i]) < 1.0e-6f;
    r.push_back(close ? 1.f : 0.f);
    n.std[1] = 0.0f;
    e.clear();
    r.push_back(!normalize_slat_f32(d, n, o, &e) && !e.empty() ? 1.f : 0.f);
    put("pipeline_utils", r);
}

SLatDecoderBlockWeightsF32 dec_block(int i, bool c2s, int C, int O, int mlp) {
    SLatDecoderBlockWeightsF32 b;
    const std::string p = "dec.b" + std::to_string(i) + ".";
    auto g = [&](const char *n) { return in.count(p + n) ? F(p + n).data() : nullptr; };
    b.kind = c2s ? SLatDecoderBlockKind::channel_to_spatial : SLatDecoderBlockKind::convnext;
    b.channels = C;
    b.out_channels = O;
    b.mlp_hidden = mlp;
    if (!c2s) {
        b.norm_weight = g("norm_w");
        b.norm_bias = g("norm_b");
        b.conv1_weight = g("conv_w");
        b.conv1_bias = g("conv_b");
        b.mlp0_weight = g("mlp0_w");
        b.mlp0_bias = g("mlp0_b");
        b.mlp2_weight = g("mlp2_w");
        b.mlp2_bias = g("mlp2_b");
    } else {
        b.norm1_weight = g("norm1_w");
        b.norm1_bias = g("norm1_b");
        b.conv1_weight = g("conv1_w");
        b.conv1_bias = g("conv1_b");
        b.conv2_weight = g("conv2_w");
        b.conv2_bias = g("conv2_b");
        b.to_subdiv_weight = g("subdiv_w");
        b.to_subdiv_bias = g("subdiv_b");
    }
    return b;
}

// The reference decoder fixture (3 levels 8 -> 8 -> 4, predicted subdivision).
void decoder() {
    SLatDecoderWeightsF32 w;
    w.from_latent_weight = F("dec.from_latent_w").data();
    w.from_latent_bias = F("dec.from_latent_b").data();
    w.output_weight = F("dec.output_w").data();
    w.output_bias = F("dec.output_b").data();
    w.blocks = {dec_block(0, false, 8, 8, 32), dec_block(1, true, 8, 8, 0), dec_block(2, false, 8, 8, 32),
                dec_block(3, true, 8, 4, 0), dec_block(4, false, 4, 4, 16)};
    SLatDecoderConfig cfg;
    cfg.latent_channels = 3;
    cfg.out_channels = 3;
    cfg.pred_subdiv = true;
    cfg.model_channels = {8, 8, 4};
    cfg.num_blocks = {1, 1, 1};
    const SparseTensorF32 x = sparse(I("dec.coords"), F("dec.x"), 3, 1, 2, 2, 2);
    SparseTensorF32 o;
    std::vector<SparseTensorF32> preds;
    std::string e;
    if (slat_decoder_forward_f32(x, cfg, w, nullptr, o, &preds, &e)) {
        put("slat_decoder_coords", o.coords);
        put("slat_decoder_output", o.feats);
        put("slat_decoder_subdiv_0_output", preds.at(0).feats);
        put("slat_decoder_subdiv_1_output", preds.at(1).feats);
    } else put_error("slat_decoder_forward", e);
    SLatDecoderModel model;
    SLatDecoderHParams hp;
    hp.latent_channels = 3;
    hp.out_channels = 3;
    hp.pred_subdiv = true;
    hp.model_channels = cfg.model_channels;
    hp.num_blocks = cfg.num_blocks;
    if (!model.bind(hp, w, &e)) {
        put_error("slat_decoder_bind", e);
        return;
    }
    for (int level = 0; level < 3; ++level) {
        if (model.upsample_coords(x, level, o, &e)) put("slat_decoder_upsample_coords_" + std::to_string(level), o.coords);
        else put_error("slat_decoder_upsample_coords", e);
    }
    if (model.decode(x, nullptr, o, &preds, &e)) put("slat_decoder_model_output", o.feats);
    else put_error("slat_decoder_decode", e);
    // single blocks on the level-0 hidden state
    const SparseTensorF32 h0 = sparse(I("dec.coords"), F("dec.h0"), 8, 1, 2, 2, 2);
    if (sparse_convnext_block_f32(h0, w.blocks[0], 1e-6f, o, &e)) put("dec_convnext_output", o.feats);
    else put_error("dec_convnext", e);
    SparseTensorF32 pred;
    if (sparse_resblock_c2s_f32(h0, w.blocks[1], 1e-6f, true, nullptr, o, &pred, &e)) {
        put("dec_c2s_coords", o.coords);
        put("dec_c2s_output", o.feats);
        put("dec_c2s_subdiv", pred.feats);
    } else put_error("dec_c2s", e);
}

void sampler() {
    const SparseTensorF32 noise = sparse(I("fs.coords"), F("fs.noise"), 3, 2, 3, 3, 3);
    FlowEulerSamplerConfig sc;
    sc.steps = 6;
    sc.sigma_min = 0.031f;
    sc.rescale_t = 2.7f;
    sc.guidance_strength = 2.35f;
    sc.guidance_rescale = 0.41f;
    sc.guidance_interval_min = 0.34f;
    sc.guidance_interval_max = 0.91f;
    sc.record_trajectory = true;
    FlowVelocityFn model = [](const SparseTensorF32 &state, float t, bool cond, SparseTensorF32 &v, std::string *) {
        v = state;
        const float cv = cond ? 0.19f : -0.07f;
        for (std::size_t p = 0; p < state.points(); ++p)
            for (int c = 0; c < state.channels; ++c) {
                const std::size_t i = p * state.channels + c;
                v.feats[i] = 0.043f * state.feats[i] + 0.00037f * t + 0.011f * static_cast<float>(c) + cv;
            }
        return true;
    };
    FlowEulerSampleF32 r;
    std::string e;
    if (flow_euler_sample_f32(noise, sc, model, r, &e)) {
        put("flow_sampler_samples", r.samples.feats);
        put("flow_sampler_pred_x_t_last", r.pred_x_t.back().feats);
        put("flow_sampler_pred_x_0_last", r.pred_x_0.back().feats);
    } else put_error("flow_sampler", e);
}

}  // namespace

int main(int argc, char **argv) {
    if (argc < 3 || argc > 5 || !read_inputs(argv[1])) {
        std::cerr << "usage: host_api_check <inputs.bin> <outputs.bin> [<flow pack.gguf> [<texture pack.gguf>]]\n";
        return 2;
    }
    out_file.open(argv[2], std::ios::binary);
    try {
        sparse_ops();
        block();
        flow();
        flow_device();
        decoder();
        sampler();
        pipeline_utils();
        if (argc >= 4) flow_gguf(argv[3]);
        if (argc >= 5) flow_concat_gguf(argv[4]);
    } catch (const std::exception &ex) {
        std::cerr << "exception: " << ex.what() << "\n";
        return 3;
    }
    out_file.close();
    std::cout << (failures ? "FAILED" : "ok") << " " << failures << "\n";
    return failures ? 1 : 0;
}
