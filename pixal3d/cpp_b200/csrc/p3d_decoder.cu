// Device-resident SLat decoder: slat_decoder_forward_f32 and
// slat_decoder_upsample_coords_f32 (src/slat_decoder.cpp:185-455) as one
// object behind the C ABI.
//
//   from_latent linear -> per level: ConvNeXt blocks (sparse conv, LayerNorm,
//   MLP with SiLU, residual) -> channel-to-spatial res block to the next,
//   2x finer level (predicted or guided subdivision, LN+SiLU, conv to 8x
//   channels, channel-to-spatial, skip = repeated input channels,
//   LN+SiLU, conv, residual) -> final LayerNorm (eps 1e-5) + output linear.
//
// Weights live on the device as 16-bit operands padded to the kernels' row
// pitch (64 for the gather-GEMM conv input, 8 for linears).  The residual
// stream is f32.  Each level's coordinates, neighbour map and predicted
// subdivision stay on the device; the only host synchronisation per level is
// reading the next level's point count.  Workspaces are grow-only pools.
#include <string>
#include <unordered_map>
#include <vector>

#include "p3d_common.cuh"

namespace {

struct DecBlock {
    int kind = 0, C = 0, out = 0, mlp = 0;
    int64_t Cp64 = 0, Ck8 = 0, mlp_p = 0, Op64 = 0;
    uint16_t *w_conv1 = nullptr, *w_conv2 = nullptr, *w_mlp0 = nullptr, *w_mlp2 = nullptr, *w_sub = nullptr;
    float *b_conv1 = nullptr, *b_conv2 = nullptr, *b_mlp0 = nullptr, *b_mlp2 = nullptr, *b_sub = nullptr;
    float *norm_w = nullptr, *norm_b = nullptr;
};

int64_t pad_to(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

}  // namespace

struct p3d_decoder {
    p3d_ctx *ctx = nullptr;
    p3d_decoder_config cfg{};
    int dt = P3D_F16;
    std::vector<void *> allocs;  // weights
    struct PoolBuf {
        void *ptr = nullptr;
        size_t bytes = 0;
    };
    std::unordered_map<std::string, PoolBuf> pool;  // workspaces, grow-only
    uint16_t *w_lat = nullptr, *w_out = nullptr;
    float *b_lat = nullptr, *b_out = nullptr;
    int64_t lat_pad = 0, last_k8 = 0;
    std::vector<DecBlock> blocks;
    // last run
    int levels_done = 0;
    std::vector<int64_t> rows;
    float *result = nullptr;

    int alloc_bytes(void **p, size_t bytes) {
        *p = nullptr;
        if (cudaMalloc(p, bytes ? bytes : 1) != cudaSuccess)
            return p3d::set_error(ctx, P3D_ERR_CUDA, "p3d_decoder: cudaMalloc failed");
        allocs.push_back(*p);
        return P3D_OK;
    }
    template <typename T>
    T *ws(const std::string &name, int64_t count) {
        PoolBuf &b = pool[name];
        const size_t bytes = sizeof(T) * static_cast<size_t>(count > 0 ? count : 1);
        if (b.bytes < bytes) {
            if (b.ptr) cudaFree(b.ptr);
            b.ptr = nullptr;
            b.bytes = 0;
            if (cudaMalloc(&b.ptr, bytes) != cudaSuccess) return nullptr;
            b.bytes = bytes;
        }
        return static_cast<T *>(b.ptr);
    }
    ~p3d_decoder() {
        for (auto &kv : pool) cudaFree(kv.second.ptr);
        for (void *p : allocs) cudaFree(p);
    }
};

using p3d::DeviceGuard;

namespace {

using p3d::set_error;

#define DEC_TRY(expr)        \
    do {                     \
        int rc_ = (expr);    \
        if (rc_) return rc_; \
    } while (0)

// f32 device [rows][cols] weights -> 16-bit [rows_pad][ld] (zero padded).
int upload_w(p3d_decoder *d, const float *src, int64_t rows, int64_t cols, int64_t rows_pad, int64_t ld,
             uint16_t **out) {
    void *p = nullptr;
    DEC_TRY(d->alloc_bytes(&p, sizeof(uint16_t) * rows_pad * ld));
    *out = static_cast<uint16_t *>(p);
    if (rows_pad > rows)
        P3D_CUDA(d->ctx, cudaMemsetAsync(*out + rows * ld, 0, sizeof(uint16_t) * (rows_pad - rows) * ld, d->ctx->stream));
    return p3d_pack_operand(d->ctx, src, rows, static_cast<int>(cols), *out, ld, d->dt);
}

// f32 device bias [n] -> f32 [n_pad] (zero padded); null -> zeros.
int upload_b(p3d_decoder *d, const float *src, int64_t n, int64_t n_pad, float **out) {
    void *p = nullptr;
    DEC_TRY(d->alloc_bytes(&p, sizeof(float) * n_pad));
    *out = static_cast<float *>(p);
    P3D_CUDA(d->ctx, cudaMemsetAsync(*out, 0, sizeof(float) * n_pad, d->ctx->stream));
    if (src) P3D_CUDA(d->ctx, cudaMemcpyAsync(*out, src, sizeof(float) * n, cudaMemcpyDeviceToDevice, d->ctx->stream));
    return P3D_OK;
}

int copy_f32(p3d_decoder *d, const float *src, int64_t n, float **out) {
    if (!src) return set_error(d->ctx, P3D_ERR_INVALID, "missing SLat decoder tensor");
    return upload_b(d, src, n, n, out);
}

int nbr_map(p3d_decoder *d, int level, const int32_t *coords, int64_t n, int32_t **nbr) {
    *nbr = d->ws<int32_t>("nbr" + std::to_string(level), 27 * n);
    const size_t wsb = p3d_neighbor_map27_workspace(n);
    void *hash = d->ws<uint8_t>("hash", static_cast<int64_t>(wsb));
    if (!*nbr || !hash) return set_error(d->ctx, P3D_ERR_CUDA, "p3d_decoder: workspace allocation failed");
    return p3d_neighbor_map27_ws(d->ctx, coords, n, hash, wsb, *nbr);
}

}  // namespace

extern "C" int p3d_decoder_create(p3d_ctx *ctx, const p3d_decoder_config *cfg, const p3d_decoder_weights *w,
                                  p3d_decoder **out) {
    if (!ctx || !cfg || !w || !out) return P3D_ERR_INVALID;
    *out = nullptr;
    DeviceGuard dg(ctx->device);
    P3D_REQUIRE(ctx, cfg->levels > 0 && cfg->levels <= P3D_DECODER_MAX_LEVELS && cfg->latent_channels > 0 &&
                         cfg->out_channels > 0 && cfg->norm_eps > 0.0f,
                "invalid SLat decoder configuration");
    int expected = cfg->levels - 1;
    for (int l = 0; l < cfg->levels; ++l) {
        P3D_REQUIRE(ctx, cfg->model_channels[l] > 0 && cfg->num_blocks[l] >= 0, "invalid SLat decoder block count");
        expected += cfg->num_blocks[l];
    }
    P3D_REQUIRE(ctx, w->blocks && w->num_blocks == expected,
                "SLat decoder weight block count does not match configuration");
    P3D_REQUIRE(ctx, w->from_latent_w && w->output_w, "missing SLat decoder tensor");
    p3d_decoder *d = new p3d_decoder();
    d->ctx = ctx;
    d->cfg = *cfg;
    d->dt = cfg->operand_dtype == P3D_BF16 ? P3D_BF16 : P3D_F16;
    auto fail = [&](int rc) {
        cudaStreamSynchronize(ctx->stream);
        delete d;
        return rc;
    };
    int rc;
    const int C0 = cfg->model_channels[0], CL = cfg->model_channels[cfg->levels - 1];
    d->lat_pad = pad_to(cfg->latent_channels, 8);
    d->last_k8 = pad_to(CL, 8);
    if ((rc = upload_w(d, w->from_latent_w, C0, cfg->latent_channels, C0, d->lat_pad, &d->w_lat))) return fail(rc);
    if ((rc = upload_b(d, w->from_latent_b, C0, C0, &d->b_lat))) return fail(rc);
    if ((rc = upload_w(d, w->output_w, cfg->out_channels, CL, cfg->out_channels, d->last_k8, &d->w_out)))
        return fail(rc);
    if ((rc = upload_b(d, w->output_b, cfg->out_channels, cfg->out_channels, &d->b_out))) return fail(rc);
    int bi = 0;
    for (int l = 0; l < cfg->levels; ++l) {
        const int C = cfg->model_channels[l];
        for (int k = 0; k <= cfg->num_blocks[l]; ++k) {
            const bool c2s = k == cfg->num_blocks[l];
            if (c2s && l + 1 == cfg->levels) break;
            const p3d_decoder_block &s = w->blocks[bi++];
            DecBlock b;
            b.kind = c2s ? 1 : 0;
            b.C = C;
            b.Cp64 = pad_to(C, 64);
            b.Ck8 = pad_to(C, 8);
            if (s.kind != b.kind || s.channels != C)
                return fail(set_error(ctx, P3D_ERR_INVALID,
                                      c2s ? "SLat decoder expected channel-to-spatial block"
                                          : "SLat decoder expected ConvNeXt block"));
            if (!c2s) {
                if (s.mlp_hidden <= 0 || s.out_channels != C || !s.conv1_w || !s.norm_w || !s.norm_b || !s.mlp0_w ||
                    !s.mlp2_w)
                    return fail(set_error(ctx, P3D_ERR_INVALID, "invalid SLat ConvNeXt block dimensions"));
                b.mlp = s.mlp_hidden;
                b.mlp_p = pad_to(b.mlp, 8);
                if ((rc = upload_w(d, s.conv1_w, 27LL * C, C, 27LL * C, b.Cp64, &b.w_conv1)) ||
                    (rc = upload_b(d, s.conv1_b, C, C, &b.b_conv1)) || (rc = copy_f32(d, s.norm_w, C, &b.norm_w)) ||
                    (rc = copy_f32(d, s.norm_b, C, &b.norm_b)) ||
                    (rc = upload_w(d, s.mlp0_w, b.mlp, C, b.mlp_p, b.Ck8, &b.w_mlp0)) ||
                    (rc = upload_b(d, s.mlp0_b, b.mlp, b.mlp_p, &b.b_mlp0)) ||
                    (rc = upload_w(d, s.mlp2_w, C, b.mlp, C, b.mlp_p, &b.w_mlp2)) ||
                    (rc = upload_b(d, s.mlp2_b, C, C, &b.b_mlp2)))
                    return fail(rc);
            } else {
                const int O = s.out_channels;
                if (O <= 0 || C % 8 != 0 || O != cfg->model_channels[l + 1] || O % (C / 8) != 0 || !s.conv1_w ||
                    !s.conv2_w || !s.norm1_w || !s.norm1_b || (cfg->pred_subdiv && !s.subdiv_w))
                    return fail(set_error(ctx, P3D_ERR_INVALID, "invalid SLat channel-to-spatial block dimensions"));
                b.out = O;
                b.Op64 = pad_to(O, 64);
                if ((rc = copy_f32(d, s.norm1_w, C, &b.norm_w)) || (rc = copy_f32(d, s.norm1_b, C, &b.norm_b)) ||
                    (rc = upload_w(d, s.conv1_w, 27LL * O * 8, C, 27LL * O * 8, b.Cp64, &b.w_conv1)) ||
                    (rc = upload_b(d, s.conv1_b, 8LL * O, 8LL * O, &b.b_conv1)) ||
                    (rc = upload_w(d, s.conv2_w, 27LL * O, O, 27LL * O, b.Op64, &b.w_conv2)) ||
                    (rc = upload_b(d, s.conv2_b, O, O, &b.b_conv2)))
                    return fail(rc);
                if (cfg->pred_subdiv && ((rc = upload_w(d, s.subdiv_w, 8, C, 8, b.Ck8, &b.w_sub)) ||
                                         (rc = upload_b(d, s.subdiv_b, 8, 8, &b.b_sub))))
                    return fail(rc);
            }
            d->blocks.push_back(b);
        }
    }
    if (cudaStreamSynchronize(ctx->stream) != cudaSuccess)
        return fail(set_error(ctx, P3D_ERR_CUDA, "p3d_decoder_create: weight upload failed"));
    *out = d;
    return P3D_OK;
}

extern "C" int p3d_decoder_destroy(p3d_decoder *d) {
    if (d) {
        DeviceGuard dg(d->ctx->device);
        cudaStreamSynchronize(d->ctx->stream);
        delete d;
    }
    return P3D_OK;
}

extern "C" int p3d_decoder_run(p3d_decoder *d, const int32_t *coords, int64_t n, int batch, int sx, int sy, int sz,
                               const float *latent, const float *const *guides, const int64_t *guide_rows,
                               int stop_level) {
    if (!d) return P3D_ERR_INVALID;
    p3d_ctx *ctx = d->ctx;
    DeviceGuard dg(ctx->device);
    const p3d_decoder_config &cfg = d->cfg;
    P3D_REQUIRE(ctx, coords && latent && n > 0 && batch > 0 && sx > 0 && sy > 0 && sz > 0,
                "p3d_decoder_run: bad argument");
    P3D_REQUIRE(ctx, stop_level >= 0 && stop_level <= cfg.levels, "p3d_decoder_run: stop level out of range");
    P3D_REQUIRE(ctx, n < (int64_t(1) << 31) / 27, "p3d_decoder_run: too many points");
    const int dt = d->dt;
    d->levels_done = 0;
    d->rows.assign(cfg.levels, 0);
    d->result = nullptr;
    // level 0 coordinates and the from_latent linear
    int32_t *lc = d->ws<int32_t>("coords0", n * 4);
    const int C0 = cfg.model_channels[0];
    uint16_t *x16 = d->ws<uint16_t>("op", n * d->lat_pad);
    float *h = d->ws<float>("h0", n * C0);
    if (!lc || !x16 || !h) return set_error(ctx, P3D_ERR_CUDA, "p3d_decoder: workspace allocation failed");
    P3D_CUDA(ctx, cudaMemcpyAsync(lc, coords, sizeof(int32_t) * n * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    DEC_TRY(p3d_pack_operand(ctx, latent, n, cfg.latent_channels, x16, d->lat_pad, dt));
    DEC_TRY(p3d_linear(ctx, x16, d->lat_pad, d->w_lat, dt, d->b_lat, n, C0, d->lat_pad, h, C0, P3D_F32, P3D_EPI_NONE,
                       nullptr, 0, nullptr, 0));
    d->rows[0] = n;
    int bi = 0;
    int32_t *nbr = nullptr;
    DEC_TRY(nbr_map(d, 0, lc, n, &nbr));
    for (int l = 0; l < cfg.levels; ++l) {
        const int C = cfg.model_channels[l];
        d->levels_done = l + 1;
        if (l == stop_level) {
            d->result = h;
            return p3d_ctx_check(ctx);
        }
        for (int k = 0; k < cfg.num_blocks[l]; ++k) {
            const DecBlock &b = d->blocks[bi++];
            // ConvNeXt (src/slat_decoder.cpp:185-222): h += mlp2(silu(mlp0(LN(conv(h)))))
            uint16_t *op = d->ws<uint16_t>("op", n * b.Cp64);
            float *t = d->ws<float>("t", n * C);
            uint16_t *ln = d->ws<uint16_t>("ln", n * b.Ck8);
            uint16_t *hid = d->ws<uint16_t>("hid", n * b.mlp_p);
            if (!op || !t || !ln || !hid) return set_error(ctx, P3D_ERR_CUDA, "p3d_decoder: workspace allocation failed");
            DEC_TRY(p3d_pack_operand(ctx, h, n, C, op, b.Cp64, dt));
            DEC_TRY(p3d_subm_conv3d(ctx, op, n, b.Cp64, nbr, b.w_conv1, dt, b.b_conv1, C, t, C, P3D_F32, P3D_EPI_NONE,
                                    nullptr, 0, nullptr, 0));
            DEC_TRY(p3d_layernorm_act(ctx, t, n, C, cfg.norm_eps, b.norm_w, b.norm_b, 0, ln, b.Ck8, dt));
            DEC_TRY(p3d_linear(ctx, ln, b.Ck8, b.w_mlp0, dt, b.b_mlp0, n, b.mlp_p, b.Ck8, hid, b.mlp_p, dt,
                               P3D_EPI_SILU, nullptr, 0, nullptr, 0));
            DEC_TRY(p3d_linear(ctx, hid, b.mlp_p, b.w_mlp2, dt, b.b_mlp2, n, C, b.mlp_p, h, C, P3D_F32,
                               P3D_EPI_RESIDUAL, nullptr, 0, nullptr, 0));
        }
        if (l + 1 == cfg.levels) break;
        // channel-to-spatial res block (src/slat_decoder.cpp:224-288)
        const DecBlock &b = d->blocks[bi++];
        const int O = b.out;
        const float *mask = nullptr;
        if (cfg.pred_subdiv) {
            uint16_t *hk = d->ws<uint16_t>("op", n * b.Ck8);
            float *sub = d->ws<float>("sub" + std::to_string(l), n * 8);
            if (!hk || !sub) return set_error(ctx, P3D_ERR_CUDA, "p3d_decoder: workspace allocation failed");
            DEC_TRY(p3d_pack_operand(ctx, h, n, C, hk, b.Ck8, dt));
            DEC_TRY(p3d_linear(ctx, hk, b.Ck8, b.w_sub, dt, b.b_sub, n, 8, b.Ck8, sub, 8, P3D_F32, P3D_EPI_NONE,
                               nullptr, 0, nullptr, 0));
            mask = sub;
        } else if (guides && guides[l]) {
            P3D_REQUIRE(ctx, guide_rows && guide_rows[l] == n, "sparse subdivision shape or coordinates do not match input");
            mask = guides[l];
        }
        uint16_t *ln1 = d->ws<uint16_t>("op", n * b.Cp64);
        float *packed = d->ws<float>("packed", n * 8 * O);
        int64_t *scratch = d->ws<int64_t>("c2s_scratch", n + 1);
        int32_t *nc = d->ws<int32_t>("coords" + std::to_string(l + 1), n * 8 * 4);
        int32_t *src_row = d->ws<int32_t>("src_row", n * 8);
        int8_t *src_child = d->ws<int8_t>("src_child", n * 8);
        int64_t *dm = d->ws<int64_t>("m", 1);
        if (!ln1 || !packed || !scratch || !nc || !src_row || !src_child || !dm)
            return set_error(ctx, P3D_ERR_CUDA, "p3d_decoder: workspace allocation failed");
        DEC_TRY(p3d_layernorm_act(ctx, h, n, C, cfg.norm_eps, b.norm_w, b.norm_b, 1, ln1, b.Cp64, dt));
        DEC_TRY(p3d_subm_conv3d(ctx, ln1, n, b.Cp64, nbr, b.w_conv1, dt, b.b_conv1, 8LL * O, packed, 8LL * O, P3D_F32,
                                P3D_EPI_NONE, nullptr, 0, nullptr, 0));
        DEC_TRY(p3d_c2s_topology(ctx, lc, n, 2, mask, scratch, nc, src_row, src_child, dm));
        int64_t m = 0;
        P3D_CUDA(ctx, cudaMemcpyAsync(&m, dm, sizeof(int64_t), cudaMemcpyDeviceToHost, ctx->stream));
        P3D_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
        DEC_TRY(p3d_ctx_check(ctx));
        P3D_REQUIRE(ctx, m > 0, "SLat decoder subdivision removed every point");
        P3D_REQUIRE(ctx, m < (int64_t(1) << 31) / 27, "p3d_decoder_run: too many points");
        float *hs = d->ws<float>("hs", m * O);
        float *hn = d->ws<float>((l & 1) ? "h0" : "h1", m * O);
        uint16_t *ln2 = d->ws<uint16_t>("op2", m * b.Op64);
        if (!hs || !hn || !ln2) return set_error(ctx, P3D_ERR_CUDA, "p3d_decoder: workspace allocation failed");
        DEC_TRY(p3d_c2s_gather(ctx, packed, 8LL * O, src_row, src_child, m, O, 1, P3D_F32, hs));
        // skip: the input's channels to space, each repeated O / (C/8) times (repeat_channels, :80-109)
        DEC_TRY(p3d_c2s_gather(ctx, h, C, src_row, src_child, m, C / 8, O / (C / 8), P3D_F32, hn));
        DEC_TRY(p3d_layernorm_act(ctx, hs, m, O, cfg.norm_eps, nullptr, nullptr, 1, ln2, b.Op64, dt));
        DEC_TRY(nbr_map(d, l + 1, nc, m, &nbr));
        DEC_TRY(p3d_subm_conv3d(ctx, ln2, m, b.Op64, nbr, b.w_conv2, dt, b.b_conv2, O, hn, O, P3D_F32,
                                P3D_EPI_RESIDUAL, nullptr, 0, nullptr, 0));
        h = hn;
        lc = nc;
        n = m;
        d->rows[l + 1] = m;
    }
    // final LayerNorm (eps 1e-5, k_slat_decoder_final_layer_norm_eps) + output linear
    const int CL = cfg.model_channels[cfg.levels - 1];
    uint16_t *lnf = d->ws<uint16_t>("ln", n * d->last_k8);
    float *res = d->ws<float>("result", n * cfg.out_channels);
    if (!lnf || !res) return set_error(ctx, P3D_ERR_CUDA, "p3d_decoder: workspace allocation failed");
    DEC_TRY(p3d_layernorm_act(ctx, h, n, CL, 1e-5f, nullptr, nullptr, 0, lnf, d->last_k8, dt));
    DEC_TRY(p3d_linear(ctx, lnf, d->last_k8, d->w_out, dt, d->b_out, n, cfg.out_channels, d->last_k8, res,
                       cfg.out_channels, P3D_F32, P3D_EPI_NONE, nullptr, 0, nullptr, 0));
    d->result = res;
    return P3D_OK;
}

extern "C" int64_t p3d_decoder_rows(const p3d_decoder *d, int level) {
    if (!d || level < 0 || level >= static_cast<int>(d->rows.size())) return -1;
    return d->rows[level];
}

extern "C" int p3d_decoder_coords(p3d_decoder *d, int level, int32_t *out) {
    if (!d || !out) return P3D_ERR_INVALID;
    p3d_ctx *ctx = d->ctx;
    P3D_REQUIRE(ctx, level >= 0 && level < d->levels_done, "p3d_decoder_coords: level not computed");
    auto it = d->pool.find("coords" + std::to_string(level));
    P3D_REQUIRE(ctx, it != d->pool.end(), "p3d_decoder_coords: level not computed");
    DeviceGuard dg(ctx->device);
    P3D_CUDA(ctx, cudaMemcpyAsync(out, it->second.ptr, sizeof(int32_t) * 4 * d->rows[level], cudaMemcpyDeviceToDevice,
                                  ctx->stream));
    return P3D_OK;
}

extern "C" int p3d_decoder_output(p3d_decoder *d, float *out) {
    if (!d || !out) return P3D_ERR_INVALID;
    p3d_ctx *ctx = d->ctx;
    P3D_REQUIRE(ctx, d->result, "p3d_decoder_output: no completed run");
    const int last = d->levels_done - 1;
    const bool stopped = d->result != d->pool["result"].ptr;
    const int64_t cols = stopped ? d->cfg.model_channels[last] : d->cfg.out_channels;
    DeviceGuard dg(ctx->device);
    P3D_CUDA(ctx, cudaMemcpyAsync(out, d->result, sizeof(float) * cols * d->rows[last], cudaMemcpyDeviceToDevice,
                                  ctx->stream));
    return P3D_OK;
}

extern "C" int p3d_decoder_subdivision(p3d_decoder *d, int level, float *out) {
    if (!d || !out) return P3D_ERR_INVALID;
    p3d_ctx *ctx = d->ctx;
    P3D_REQUIRE(ctx, d->cfg.pred_subdiv && level >= 0 && level + 1 < d->levels_done,
                "p3d_decoder_subdivision: no predicted subdivision at this level");
    auto it = d->pool.find("sub" + std::to_string(level));
    P3D_REQUIRE(ctx, it != d->pool.end(), "p3d_decoder_subdivision: no predicted subdivision at this level");
    DeviceGuard dg(ctx->device);
    P3D_CUDA(ctx, cudaMemcpyAsync(out, it->second.ptr, sizeof(float) * 8 * d->rows[level], cudaMemcpyDeviceToDevice,
                                  ctx->stream));
    return P3D_OK;
}
