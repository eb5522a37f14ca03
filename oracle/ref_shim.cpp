// extern "C" shim over the reference's own CPU F32 path (Pixal3D.cpp).
//
// TEST INFRASTRUCTURE ONLY.  Linked with the reference sources into
// oracle/_ref/libp3dref.so by oracle/Makefile.  Used by tests/ (to pin the
// numpy restatement in oracle/oracle.py) and by bench.py's CPU-baseline leg.
// It is never part of the product path.
//
// Every function builds the reference's SparseTensorF32 / VarLenTensorF32
// from plain arrays, calls the reference function named in its comment, and
// copies the result back.  Return value: 0 on success, 1 when the reference
// returned false (its error string is copied into err).

#include "pixal3d/cpu_threads.h"
#include "pixal3d/flow.h"
#include "pixal3d/flow_sampler.h"
#include "pixal3d/projection.h"
#include "pixal3d/slat_decoder.h"
#include "pixal3d/slat_flow.h"
#include "pixal3d/sparse.h"
#include "pixal3d/sparse_transformer.h"

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

namespace pixal3d {
// Defined in the extracted decoder translation unit (oracle/Makefile).
bool p3dref_reference_neighbor_map(const SparseTensorF32 & input,
                                   std::vector<std::int32_t> & out, std::string * error);
std::uint64_t p3dref_coords_fingerprint(const std::vector<std::int32_t> & coords);
}  // namespace pixal3d

namespace pixal3d {
// src/pipeline.cpp glue built from the extracted translation unit (the
// reference's include/pixal3d/pipeline.h pulls in ggml through ss_flow.h,
// so its two declarations used here are repeated).
struct SLatNormalizationF32 {
    std::vector<float> mean;
    std::vector<float> std;
};
bool normalize_slat_f32(const SparseTensorF32 & input, const SLatNormalizationF32 & normalization,
                        SparseTensorF32 & output, std::string * error);
bool quantize_slat_coords_f32(const SparseTensorF32 & upsampled_coords, int low_resolution,
                              int requested_resolution, std::size_t max_num_tokens,
                              std::vector<std::int32_t> & coords, int & actual_resolution, std::string * error);
}  // namespace pixal3d

using namespace pixal3d;

namespace {

struct P3dRefShape {
    int batch;
    int sx, sy, sz;
};

SparseTensorF32 make_sparse(const int32_t * coords, int64_t n, const float * feats, int channels,
                            int batch, int sx, int sy, int sz) {
    SparseTensorF32 t;
    t.batch_size = batch;
    t.channels = channels;
    t.spatial_x = sx;
    t.spatial_y = sy;
    t.spatial_z = sz;
    t.coords.assign(coords, coords + n * 4);
    if (feats) t.feats.assign(feats, feats + n * static_cast<int64_t>(channels));
    else t.feats.assign(static_cast<size_t>(n) * channels, 0.0f);
    return t;
}

VarLenTensorF32 make_varlen(const int64_t * offsets, int batch, const float * feats, int channels) {
    VarLenTensorF32 t;
    t.batch_size = batch;
    t.channels = channels;
    t.offsets.resize(batch + 1);
    for (int i = 0; i <= batch; ++i) t.offsets[i] = static_cast<size_t>(offsets[i]);
    t.feats.assign(feats, feats + offsets[batch] * channels);
    return t;
}

int fail(const std::string & e, char * err, int errlen) {
    if (err && errlen > 0) {
        std::strncpy(err, e.c_str(), errlen - 1);
        err[errlen - 1] = 0;
    }
    return 1;
}

void copy_out(const std::vector<float> & v, float * out) { std::memcpy(out, v.data(), v.size() * 4); }

SparseTransformerBlockWeightsF32 block_weights(const float * const * p) {
    SparseTransformerBlockWeightsF32 w;
    w.modulation = p[0];
    w.self_to_qkv_weight = p[1];
    w.self_to_qkv_bias = p[2];
    w.self_q_gamma = p[3];
    w.self_k_gamma = p[4];
    w.self_to_out_weight = p[5];
    w.self_to_out_bias = p[6];
    w.norm2_weight = p[7];
    w.norm2_bias = p[8];
    w.cross_to_q_weight = p[9];
    w.cross_to_q_bias = p[10];
    w.cross_to_kv_weight = p[11];
    w.cross_to_kv_bias = p[12];
    w.cross_q_gamma = p[13];
    w.cross_k_gamma = p[14];
    w.cross_to_out_weight = p[15];
    w.cross_to_out_bias = p[16];
    w.proj_weight = p[17];
    w.proj_bias = p[18];
    w.mlp0_weight = p[19];
    w.mlp0_bias = p[20];
    w.mlp2_weight = p[21];
    w.mlp2_bias = p[22];
    return w;
}

// ProjectionCamera from plain values (include/pixal3d/projection.h:13-27).
ProjectionCamera make_camera(float angle, float distance, float mesh_scale, int has_transform, const float * m16) {
    ProjectionCamera cam = ProjectionCamera::front(angle, distance, mesh_scale);
    if (has_transform) {
        cam.has_transform = true;
        for (int i = 0; i < 16; ++i) cam.transform_matrix[static_cast<size_t>(i)] = m16[i];
    }
    return cam;
}

}  // namespace

extern "C" {

// pixal3d::set_cpu_thread_override (include/pixal3d/cpu_threads.h:31)
int p3dref_set_threads(int threads) { return set_cpu_thread_override(threads) ? 0 : 1; }
int p3dref_thread_count(void) { return cpu_thread_count(); }

// SparseTensorF32::valid (src/sparse.cpp:241-335)
int p3dref_valid(const int32_t * coords, int64_t n, const float * feats, int channels, int batch,
                 int sx, int sy, int sz, char * err, int errlen) {
    std::string e;
    SparseTensorF32 t = make_sparse(coords, n, feats, channels, batch, sx, sy, sz);
    return t.valid(&e) ? 0 : fail(e, err, errlen);
}

// sparse_linear (src/sparse.cpp:337-451)
int p3dref_sparse_linear(const int32_t * coords, int64_t n, const float * feats, int cin, int batch,
                         int sx, int sy, int sz, const float * w, const float * b, int cout,
                         float * out, char * err, int errlen) {
    std::string e;
    SparseTensorF32 in = make_sparse(coords, n, feats, cin, batch, sx, sy, sz), o;
    if (!sparse_linear(in, w, b, cout, o, &e)) return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

// varlen_linear (src/sparse.cpp:453-488)
int p3dref_varlen_linear(const int64_t * offsets, int batch, const float * feats, int cin,
                         const float * w, const float * b, int cout, float * out, char * err,
                         int errlen) {
    std::string e;
    VarLenTensorF32 in = make_varlen(offsets, batch, feats, cin), o;
    if (!varlen_linear(in, w, b, cout, o, &e)) return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

// sparse_layer_norm (src/sparse.cpp:490-534)
int p3dref_layer_norm(const int32_t * coords, int64_t n, const float * feats, int c, int batch,
                      int sx, int sy, int sz, float eps, const float * gamma, const float * beta,
                      float * out, char * err, int errlen) {
    std::string e;
    SparseTensorF32 in = make_sparse(coords, n, feats, c, batch, sx, sy, sz), o;
    if (!sparse_layer_norm(in, eps, gamma, beta, o, &e)) return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

// sparse_downsample_mean (src/sparse.cpp:536-602).  out_coords/out_feats must
// hold n rows; *out_n receives the output row count.
int p3dref_downsample_mean(const int32_t * coords, int64_t n, const float * feats, int c, int batch,
                           int sx, int sy, int sz, int factor, int32_t * out_coords,
                           float * out_feats, int64_t * out_n, int * out_shape, char * err,
                           int errlen) {
    std::string e;
    SparseTensorF32 in = make_sparse(coords, n, feats, c, batch, sx, sy, sz), o;
    if (!sparse_downsample_mean(in, factor, o, &e)) return fail(e, err, errlen);
    std::memcpy(out_coords, o.coords.data(), o.coords.size() * 4);
    copy_out(o.feats, out_feats);
    *out_n = static_cast<int64_t>(o.points());
    out_shape[0] = o.spatial_x;
    out_shape[1] = o.spatial_y;
    out_shape[2] = o.spatial_z;
    return 0;
}

// sparse_channel_to_spatial (src/sparse.cpp:604-702).  subdiv may be null.
// out buffers must hold n*factor^3 rows.
int p3dref_channel_to_spatial(const int32_t * coords, int64_t n, const float * feats, int c,
                              int batch, int sx, int sy, int sz, int factor, const float * subdiv,
                              int32_t * out_coords, float * out_feats, int64_t * out_n,
                              char * err, int errlen) {
    std::string e;
    SparseTensorF32 in = make_sparse(coords, n, feats, c, batch, sx, sy, sz), o, sd;
    const SparseTensorF32 * psd = nullptr;
    if (subdiv) {
        sd = make_sparse(coords, n, subdiv, factor * factor * factor, batch, sx, sy, sz);
        psd = &sd;
    }
    if (!sparse_channel_to_spatial(in, factor, psd, o, &e)) return fail(e, err, errlen);
    std::memcpy(out_coords, o.coords.data(), o.coords.size() * 4);
    copy_out(o.feats, out_feats);
    *out_n = static_cast<int64_t>(o.points());
    return 0;
}

// sparse_scaled_dot_product_attention (src/sparse.cpp:704-783).  Q, K and V
// rows share one coordinate list here (self-attention).
int p3dref_sdpa(const int32_t * coords, int64_t n, int batch, int sx, int sy, int sz,
                const float * q, const float * k, const float * v, int heads, int head_dim,
                int v_channels, float scale, float * out, char * err, int errlen) {
    std::string e;
    const int c = heads * head_dim;
    SparseTensorF32 tq = make_sparse(coords, n, q, c, batch, sx, sy, sz);
    SparseTensorF32 tk = make_sparse(coords, n, k, c, batch, sx, sy, sz);
    SparseTensorF32 tv = make_sparse(coords, n, v, v_channels, batch, sx, sy, sz), o;
    if (!sparse_scaled_dot_product_attention(tq, tk, tv, heads, head_dim, scale, o, &e))
        return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

// sparse_cross_attention (src/sparse.cpp:785-859)
int p3dref_cross_attention(const int32_t * coords, int64_t n, int batch, int sx, int sy, int sz,
                           const float * q, const int64_t * offsets, const float * k,
                           const float * v, int heads, int head_dim, int v_channels, float scale,
                           float * out, char * err, int errlen) {
    std::string e;
    const int c = heads * head_dim;
    SparseTensorF32 tq = make_sparse(coords, n, q, c, batch, sx, sy, sz), o;
    VarLenTensorF32 tk = make_varlen(offsets, batch, k, c);
    VarLenTensorF32 tv = make_varlen(offsets, batch, v, v_channels);
    if (!sparse_cross_attention(tq, tk, tv, heads, head_dim, scale, o, &e))
        return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

// sparse_rotary_position_embedding (src/sparse.cpp:861-917)
int p3dref_rope(const int32_t * coords, int64_t n, int batch, int sx, int sy, int sz,
                const float * feats, int heads, int head_dim, float fmin, float fbase, float * out,
                char * err, int errlen) {
    std::string e;
    SparseTensorF32 in = make_sparse(coords, n, feats, heads * head_dim, batch, sx, sy, sz), o;
    if (!sparse_rotary_position_embedding(in, heads, head_dim, fmin, fbase, o, &e))
        return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

// sparse_multihead_rms_norm (src/sparse.cpp:919-954)
int p3dref_rms_norm(const int32_t * coords, int64_t n, int batch, int sx, int sy, int sz,
                    const float * feats, int heads, int head_dim, const float * gamma, float * out,
                    char * err, int errlen) {
    std::string e;
    SparseTensorF32 in = make_sparse(coords, n, feats, heads * head_dim, batch, sx, sy, sz), o;
    if (!sparse_multihead_rms_norm(in, heads, head_dim, gamma, o, &e)) return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

// varlen_multihead_rms_norm (src/sparse.cpp:956-997)
int p3dref_varlen_rms_norm(const int64_t * offsets, int batch, const float * feats, int heads,
                           int head_dim, const float * gamma, float * out, char * err,
                           int errlen) {
    std::string e;
    VarLenTensorF32 in = make_varlen(offsets, batch, feats, heads * head_dim), o;
    if (!varlen_multihead_rms_norm(in, heads, head_dim, gamma, o, &e)) return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

// sparse_submanifold_conv3d (src/sparse.cpp:999-1055)
int p3dref_subm_conv3d(const int32_t * coords, int64_t n, const float * feats, int cin, int batch,
                       int sx, int sy, int sz, const float * w, const float * b, int cout,
                       float * out, char * err, int errlen) {
    std::string e;
    SparseTensorF32 in = make_sparse(coords, n, feats, cin, batch, sx, sy, sz), o;
    if (!sparse_submanifold_conv3d(in, w, b, cout, o, &e)) return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

// build_reference_neighbor_gather_map (src/slat_decoder.cpp:670-714);
// layout [27][n], sentinel n.
int p3dref_neighbor_map27(const int32_t * coords, int64_t n, int batch, int sx, int sy, int sz,
                          int32_t * out, char * err, int errlen) {
    std::string e;
    SparseTensorF32 in = make_sparse(coords, n, nullptr, 1, batch, sx, sy, sz);
    std::vector<int32_t> map;
    if (!p3dref_reference_neighbor_map(in, map, &e)) return fail(e, err, errlen);
    std::memcpy(out, map.data(), map.size() * 4);
    return 0;
}

// decoder_coords_fingerprint (src/slat_decoder.cpp:522-534)
uint64_t p3dref_coords_fingerprint(const int32_t * coords, int64_t n) {
    std::vector<int32_t> v(coords, coords + n * 4);
    return pixal3d::p3dref_coords_fingerprint(v);
}

// timestep_embed_mlp (src/flow.cpp:125-180)
int p3dref_timestep_embed_mlp(const float * t, int64_t batch, int hidden, int freq,
                              const float * w0, const float * b0, const float * w2,
                              const float * b2, float * out, char * err, int errlen) {
    std::string e;
    std::vector<float> o;
    if (!timestep_embed_mlp(t, batch, hidden, freq, w0, b0, w2, b2, o, &e))
        return fail(e, err, errlen);
    copy_out(o, out);
    return 0;
}

// sparse_transformer_cross_block_f32 (src/sparse_transformer.cpp:138-292).
// cfg_i = {channels, heads, mlp_hidden, ctx_channels, proj_in, use_rope,
// qk_rms, qk_rms_cross, use_proj}; cfg_f = {norm_eps, rope_fmin, rope_fbase};
// wptr = 23 pointers in SparseTransformerBlockWeightsF32 field order.
int p3dref_transformer_block(const int32_t * coords, int64_t n, int batch, int sx, int sy, int sz,
                             const float * feats, const float * tmod, const int64_t * ctx_offsets,
                             const float * ctx, const float * proj, const int * cfg_i,
                             const float * cfg_f, const float * const * wptr, float * out,
                             char * err, int errlen) {
    std::string e;
    SparseTransformerBlockConfig cfg;
    cfg.channels = cfg_i[0];
    cfg.num_heads = cfg_i[1];
    cfg.mlp_hidden = cfg_i[2];
    cfg.context_channels = cfg_i[3];
    cfg.proj_in_channels = cfg_i[4];
    cfg.use_rope = cfg_i[5] != 0;
    cfg.qk_rms_norm = cfg_i[6] != 0;
    cfg.qk_rms_norm_cross = cfg_i[7] != 0;
    cfg.use_projection = cfg_i[8] != 0;
    cfg.norm_eps = cfg_f[0];
    cfg.rope_freq_min = cfg_f[1];
    cfg.rope_freq_base = cfg_f[2];
    SparseTensorF32 in = make_sparse(coords, n, feats, cfg.channels, batch, sx, sy, sz), o, pj;
    VarLenTensorF32 g = make_varlen(ctx_offsets, batch, ctx, cfg.context_channels);
    const SparseTensorF32 * ppj = nullptr;
    if (proj) {
        pj = make_sparse(coords, n, proj, cfg.proj_in_channels, batch, sx, sy, sz);
        ppj = &pj;
    }
    if (!sparse_transformer_cross_block_f32(in, tmod, g, ppj, cfg, block_weights(wptr), o, &e))
        return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

namespace {
SLatFlowHParams flow_hparams(const int * hp_i, const float * hp_f) {
    SLatFlowHParams hp;
    hp.resolution = hp_i[0];
    hp.in_channels = hp_i[1];
    hp.out_channels = hp_i[2];
    hp.model_channels = hp_i[3];
    hp.cond_channels = hp_i[4];
    hp.num_blocks = hp_i[5];
    hp.num_heads = hp_i[6];
    hp.proj_in_channels = hp_i[7];
    hp.image_attn_mode = hp_i[8] ? "proj" : "cross";
    hp.qk_rms_norm = hp_i[9] != 0;
    hp.qk_rms_norm_cross = hp_i[10] != 0;
    hp.share_mod = true;
    hp.pe_mode = "rope";
    hp.mlp_ratio = hp_f[0];
    hp.norm_eps = hp_f[1];
    hp.rope_freq_min = hp_f[2];
    hp.rope_freq_base = hp_f[3];
    return hp;
}

SLatFlowWeightsF32 flow_weights(const float * const * top, const float * const * blocks, int nb) {
    SLatFlowWeightsF32 w;
    w.input_weight = top[0];
    w.input_bias = top[1];
    w.timestep_weight0 = top[2];
    w.timestep_bias0 = top[3];
    w.timestep_weight2 = top[4];
    w.timestep_bias2 = top[5];
    w.modulation_weight = top[6];
    w.modulation_bias = top[7];
    w.output_weight = top[8];
    w.output_bias = top[9];
    for (int i = 0; i < nb; ++i) w.blocks.push_back(block_weights(blocks + 23 * i));
    return w;
}
}  // namespace

// slat_flow_forward_f32 (src/slat_flow.cpp:161-249).
// hp_i = {resolution, in, out, model, cond, blocks, heads, proj_in, proj_mode,
// qk_rms, qk_rms_cross}; hp_f = {mlp_ratio, norm_eps, rope_fmin, rope_fbase};
// top = 10 pointers in SLatFlowWeightsF32 order; blocks = nblocks*23 pointers.
int p3dref_slat_flow_forward(const int32_t * coords, int64_t n, int batch, int sx, int sy, int sz,
                             const float * feats, const float * timesteps,
                             const int64_t * ctx_offsets, const float * ctx, const float * proj,
                             const int * hp_i, const float * hp_f, const float * const * top,
                             const float * const * blocks, float * out, char * err, int errlen) {
    std::string e;
    SLatFlowHParams hp = flow_hparams(hp_i, hp_f);
    SLatFlowWeightsF32 w = flow_weights(top, blocks, hp.num_blocks);
    SparseTensorF32 in = make_sparse(coords, n, feats, hp.in_channels, batch, sx, sy, sz), o, pj;
    VarLenTensorF32 g = make_varlen(ctx_offsets, batch, ctx, hp.cond_channels);
    const SparseTensorF32 * ppj = nullptr;
    if (proj) {
        pj = make_sparse(coords, n, proj, hp.proj_in_channels, batch, sx, sy, sz);
        ppj = &pj;
    }
    if (!slat_flow_forward_f32(in, timesteps, static_cast<size_t>(batch), g, ppj, hp, w, o, &e))
        return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

// flow_euler_sample_f32 (src/flow_sampler.cpp:245-343) driven by
// slat_flow_forward_f32 with the zeros negative condition that
// SLatFlowModel::sample builds (src/slat_flow.cpp:1401-1447).
// sc_f = {sigma_min, rescale_t, guidance, guidance_rescale, gmin, gmax};
// out_x0_last (optional) receives the last pred_x_0 (record_trajectory).
int p3dref_slat_flow_sample(const int32_t * coords, int64_t n, int batch, int sx, int sy, int sz,
                            const float * noise, const int64_t * ctx_offsets, const float * ctx,
                            const float * proj, const int * hp_i, const float * hp_f,
                            const float * const * top, const float * const * blocks, int steps,
                            const float * sc_f, float * out, float * out_x0_last, char * err,
                            int errlen) {
    std::string e;
    SLatFlowHParams hp = flow_hparams(hp_i, hp_f);
    SLatFlowWeightsF32 w = flow_weights(top, blocks, hp.num_blocks);
    SparseTensorF32 in = make_sparse(coords, n, noise, hp.in_channels, batch, sx, sy, sz), pj, npj;
    VarLenTensorF32 g = make_varlen(ctx_offsets, batch, ctx, hp.cond_channels);
    VarLenTensorF32 ng = g;
    std::fill(ng.feats.begin(), ng.feats.end(), 0.0f);
    const SparseTensorF32 * ppj = nullptr;
    const SparseTensorF32 * pnpj = nullptr;
    if (proj) {
        pj = make_sparse(coords, n, proj, hp.proj_in_channels, batch, sx, sy, sz);
        npj = pj;
        std::fill(npj.feats.begin(), npj.feats.end(), 0.0f);
        ppj = &pj;
        pnpj = &npj;
    }
    FlowEulerSamplerConfig sc;
    sc.steps = steps;
    sc.sigma_min = sc_f[0];
    sc.rescale_t = sc_f[1];
    sc.guidance_strength = sc_f[2];
    sc.guidance_rescale = sc_f[3];
    sc.guidance_interval_min = sc_f[4];
    sc.guidance_interval_max = sc_f[5];
    sc.record_trajectory = out_x0_last != nullptr;
    FlowVelocityFn cb = [&](const SparseTensorF32 & state, float t, bool cond,
                            SparseTensorF32 & vel, std::string * cerr) {
        std::vector<float> tb(static_cast<size_t>(state.batch_size), t);
        return slat_flow_forward_f32(state, tb.data(), tb.size(), cond ? g : ng, cond ? ppj : pnpj,
                                     hp, w, vel, cerr);
    };
    FlowEulerSampleF32 res;
    if (!flow_euler_sample_f32(in, sc, cb, res, &e)) return fail(e, err, errlen);
    copy_out(res.samples.feats, out);
    if (out_x0_last) copy_out(res.pred_x_0.back().feats, out_x0_last);
    return 0;
}

// flow_euler_sample_f32 (src/flow_sampler.cpp:245-343) with a C velocity
// callback: int cb(void* user, const float* state, int64_t n, int channels,
// float model_t, int conditional, float* velocity) returning 0 on success.
typedef int (*p3dref_velocity_fn)(void *, const float *, int64_t, int, float, int, float *);
int p3dref_flow_euler_sample(const int32_t * coords, int64_t n, int batch, int sx, int sy, int sz,
                             const float * noise, int channels, int steps, const float * sc_f,
                             p3dref_velocity_fn fn, void * user, float * out, char * err,
                             int errlen) {
    std::string e;
    SparseTensorF32 in = make_sparse(coords, n, noise, channels, batch, sx, sy, sz);
    FlowEulerSamplerConfig sc;
    sc.steps = steps;
    sc.sigma_min = sc_f[0];
    sc.rescale_t = sc_f[1];
    sc.guidance_strength = sc_f[2];
    sc.guidance_rescale = sc_f[3];
    sc.guidance_interval_min = sc_f[4];
    sc.guidance_interval_max = sc_f[5];
    FlowVelocityFn cb = [&](const SparseTensorF32 & state, float t, bool cond,
                            SparseTensorF32 & vel, std::string * cerr) {
        vel = state;
        if (fn(user, state.feats.data(), static_cast<int64_t>(state.points()), state.channels, t,
               cond ? 1 : 0, vel.feats.data()) != 0) {
            if (cerr) *cerr = "velocity callback failed";
            return false;
        }
        return true;
    };
    FlowEulerSampleF32 res;
    if (!flow_euler_sample_f32(in, sc, cb, res, &e)) return fail(e, err, errlen);
    copy_out(res.samples.feats, out);
    return 0;
}

// sparse_convnext_block_f32 (src/slat_decoder.cpp:185-222).
// w = {norm_w, norm_b, conv_w, conv_b, mlp0_w, mlp0_b, mlp2_w, mlp2_b}.
int p3dref_convnext_block(const int32_t * coords, int64_t n, int batch, int sx, int sy, int sz,
                          const float * feats, int channels, int mlp_hidden,
                          const float * const * w, float eps, float * out, char * err,
                          int errlen) {
    std::string e;
    SLatDecoderBlockWeightsF32 bw;
    bw.kind = SLatDecoderBlockKind::convnext;
    bw.channels = channels;
    bw.out_channels = channels;
    bw.mlp_hidden = mlp_hidden;
    bw.norm_weight = w[0];
    bw.norm_bias = w[1];
    bw.conv1_weight = w[2];
    bw.conv1_bias = w[3];
    bw.mlp0_weight = w[4];
    bw.mlp0_bias = w[5];
    bw.mlp2_weight = w[6];
    bw.mlp2_bias = w[7];
    SparseTensorF32 in = make_sparse(coords, n, feats, channels, batch, sx, sy, sz), o;
    if (!sparse_convnext_block_f32(in, bw, eps, o, &e)) return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

// sparse_resblock_c2s_f32 (src/slat_decoder.cpp:224-288).
// w = {norm1_w, norm1_b, conv1_w, conv1_b, conv2_w, conv2_b, subdiv_w, subdiv_b}.
// subdiv (optional) = guide logits [n,8]; pred (optional) receives [n,8].
// Output buffers must hold 8*n rows.
int p3dref_resblock_c2s(const int32_t * coords, int64_t n, int batch, int sx, int sy, int sz,
                        const float * feats, int channels, int out_channels,
                        const float * const * w, float eps, int pred_subdiv,
                        const float * subdiv, int32_t * out_coords, float * out_feats,
                        int64_t * out_n, float * pred, char * err, int errlen) {
    std::string e;
    SLatDecoderBlockWeightsF32 bw;
    bw.kind = SLatDecoderBlockKind::channel_to_spatial;
    bw.channels = channels;
    bw.out_channels = out_channels;
    bw.norm1_weight = w[0];
    bw.norm1_bias = w[1];
    bw.conv1_weight = w[2];
    bw.conv1_bias = w[3];
    bw.conv2_weight = w[4];
    bw.conv2_bias = w[5];
    bw.to_subdiv_weight = w[6];
    bw.to_subdiv_bias = w[7];
    SparseTensorF32 in = make_sparse(coords, n, feats, channels, batch, sx, sy, sz), o, sd, pr;
    const SparseTensorF32 * psd = nullptr;
    if (subdiv) {
        sd = make_sparse(coords, n, subdiv, 8, batch, sx, sy, sz);
        psd = &sd;
    }
    if (!sparse_resblock_c2s_f32(in, bw, eps, pred_subdiv != 0, psd, o, pred ? &pr : nullptr, &e))
        return fail(e, err, errlen);
    std::memcpy(out_coords, o.coords.data(), o.coords.size() * 4);
    copy_out(o.feats, out_feats);
    *out_n = static_cast<int64_t>(o.points());
    if (pred && pred_subdiv) copy_out(pr.feats, pred);
    return 0;
}

// project_grid_features_at_coords (src/projection.cpp:359-434): feats [n][c], valid [n].
int p3dref_project_at_coords(const float * fmap, int h, int w, int c, int grid_resolution, int image_resolution,
                             float angle, float distance, float mesh_scale, int has_transform, const float * m16,
                             const int32_t * coords, int64_t n, float * feats, uint8_t * valid, char * err,
                             int errlen) {
    ProjectionGridOptions opt;
    opt.grid_resolution = grid_resolution;
    opt.image_resolution = image_resolution;
    std::vector<std::int32_t> cv(coords, coords + 4 * n);
    std::vector<float> f;
    std::vector<std::uint8_t> v;
    std::string e;
    if (!project_grid_features_at_coords(fmap, h, w, c, opt, make_camera(angle, distance, mesh_scale, has_transform, m16),
                                         cv, f, v, &e))
        return fail(e, err, errlen);
    copy_out(f, feats);
    std::memcpy(valid, v.data(), v.size());
    return 0;
}

// project_grid_features_average (src/projection.cpp:436-481) over nviews maps
// of one shape: feats [r^3][c], valid [r^3].  cams: [nviews][4] (angle,
// distance, mesh_scale, has_transform), m16: [nviews][16].
int p3dref_project_average(const float * const * fmaps, int nviews, int h, int w, int c, int grid_resolution,
                           int image_resolution, const float * cams, const float * m16, float * feats,
                           uint8_t * valid, char * err, int errlen) {
    ProjectionGridOptions opt;
    opt.grid_resolution = grid_resolution;
    opt.image_resolution = image_resolution;
    std::vector<ProjectionView> views;
    for (int i = 0; i < nviews; ++i) {
        ProjectionView view;
        view.feature_map = fmaps[i];
        view.height = h;
        view.width = w;
        view.channels = c;
        view.camera = make_camera(cams[4 * i], cams[4 * i + 1], cams[4 * i + 2], cams[4 * i + 3] != 0.0f, m16 + 16 * i);
        views.push_back(view);
    }
    ProjectedGrid g;
    std::string e;
    if (!project_grid_features_average(views, opt, g, &e)) return fail(e, err, errlen);
    copy_out(g.features, feats);
    std::memcpy(valid, g.valid.data(), g.valid.size());
    return 0;
}

// compute_relative_calc_matrices (src/projection.cpp:528-561): relative [n][16].
int p3dref_relative_matrices(const float * c2w, const float * distances, int n, float * relative, char * err,
                             int errlen) {
    std::vector<std::array<float, 16>> m(static_cast<size_t>(n)), out;
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < 16; ++j) m[static_cast<size_t>(i)][static_cast<size_t>(j)] = c2w[16 * i + j];
    std::vector<float> d(distances, distances + n);
    std::string e;
    if (!compute_relative_calc_matrices(m, d, out, &e)) return fail(e, err, errlen);
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < 16; ++j) relative[16 * i + j] = out[static_cast<size_t>(i)][static_cast<size_t>(j)];
    return 0;
}

// normalize_slat_f32 (src/pipeline.cpp:333-358): out [n][c].
int p3dref_normalize_slat(const int32_t * coords, int64_t n, const float * feats, int c, int batch, int sx, int sy,
                          int sz, const float * mean, const float * stdv, float * out, char * err, int errlen) {
    SparseTensorF32 in = make_sparse(coords, n, feats, c, batch, sx, sy, sz);
    SLatNormalizationF32 norm;
    norm.mean.assign(mean, mean + c);
    norm.std.assign(stdv, stdv + c);
    SparseTensorF32 o;
    std::string e;
    if (!normalize_slat_f32(in, norm, o, &e)) return fail(e, err, errlen);
    copy_out(o.feats, out);
    return 0;
}

// quantize_slat_coords_f32 (src/pipeline.cpp:437-468): out [m][4], *m.
int p3dref_quantize_slat_coords(const int32_t * coords, int64_t n, int batch, int sx, int low_resolution,
                                int requested_resolution, int64_t max_tokens, int32_t * out, int64_t * m, char * err,
                                int errlen) {
    std::vector<float> zeros(static_cast<size_t>(n), 0.0f);
    SparseTensorF32 in = make_sparse(coords, n, zeros.data(), 1, batch, sx, sx, sx);
    std::vector<std::int32_t> q;
    int res = 0;
    std::string e;
    if (!quantize_slat_coords_f32(in, low_resolution, requested_resolution, static_cast<std::size_t>(max_tokens), q,
                                  res, &e))
        return fail(e, err, errlen);
    std::memcpy(out, q.data(), q.size() * 4);
    *m = static_cast<int64_t>(q.size() / 4);
    return 0;
}

}  // extern "C"
