// Projection conditioning: per-voxel camera projection and bilinear sampling
// of image feature maps (the producer of image_attn_mode=proj, reference
// src/projection.cpp).
//
// For each point (a sparse (0, x, y, z) row, or every cell of the dense
// grid in meshgrid "ij" order) and each view:
//   grid cell -> [-1, 1]^3 -> (x, -z, y) * 1 / (2 mesh_scale)   (:293-298)
//   camera space by the inverse camera-to-world matrix, perspective divide by
//   (-z_cam + 1e-8), pixel = focal_px * ndc + res/2               (:116-146)
//   grid_sample bilinear, align_corners=False, border padding     (:155-203)
// and, over views, the f32 sum in view order times 1/views (:436-481,
// src/condition.cpp:878-940); valid = projected inside the image and in
// front of the camera in at least one view.
//
// The arithmetic is IEEE single precision in the reference's operation
// order with contraction disabled (explicit _rn intrinsics), so features and
// validity flags equal the reference's CPU results bit for bit.
//
// Layout: one warp per point.  Lane v < views computes view v's geometry
// (pixel, corner rows, weights); the warp then walks the channels in tiles of
// 32 lanes x 4 (float4 loads of the four corner rows, which sit in L2: a
// 37 x 37 x 1024 map is 5.6 MB) and writes f32 or 16-bit rows.  The bound is
// the output write plus the corner reads from L2.
#include <algorithm>
#include <cmath>
#include <utility>

#include "p3d_common.cuh"

namespace p3d {
namespace {

constexpr int kMaxViews = 8;
constexpr int kProjWarps = 8;  // warps (points in flight) per block

struct ViewConst {
    const float *fmap;
    int h, w;
    float w2c[12];  // rows 0..2 of the world-to-camera matrix
    float scale, focal_px, half, res;
};

struct ProjParams {
    ViewConst view[kMaxViews];
    int nviews, grid, channels, out_dtype;
    const int32_t *coords;  // [n][4] or null (dense grid)
    int64_t n, ldo;
    void *out;
    uint8_t *valid;
    float inv_views;
    int *fault;
};

__device__ __forceinline__ float grid_base(int i, int r) {
    if (r == 1) return 0.0f;
    return __fadd_rn(-1.0f, __fdiv_rn(__fmul_rn(2.0f, static_cast<float>(i)), static_cast<float>(r - 1)));
}

// std::max(0, std::min(v, hi)): a NaN ends at 0, like the reference.
__device__ __forceinline__ float clamp_ref(float v, float hi) {
    const float t = (hi < v) ? hi : v;
    return (0.0f < t) ? t : 0.0f;
}

struct Corner {
    int64_t top, bottom;  // element offsets of rows y0, y1
    int x0, x1;           // column indices
    float wx, wy;
    bool valid;
};

__device__ __forceinline__ Corner view_geometry(const ViewConst &v, float bx, float by, float bz) {
    const float x = __fmul_rn(bx, v.scale);
    const float y = __fmul_rn(-bz, v.scale);
    const float z = __fmul_rn(by, v.scale);
    const float *m = v.w2c;
    const float xc = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(m[0], x), __fmul_rn(m[1], y)), __fmul_rn(m[2], z)), m[3]);
    const float yc = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(m[4], x), __fmul_rn(m[5], y)), __fmul_rn(m[6], z)), m[7]);
    const float zc =
        __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(m[8], x), __fmul_rn(m[9], y)), __fmul_rn(m[10], z)), m[11]);
    const float depth = -zc;
    const float den = __fadd_rn(-zc, 1e-8f);
    const float xn = __fdiv_rn(__fmul_rn(v.focal_px, xc), den);
    const float yn = __fdiv_rn(__fmul_rn(v.focal_px, yc), den);
    const float xp = __fadd_rn(xn, v.half);
    const float yp = __fadd_rn(-yn, v.half);
    Corner c;
    c.valid = xp >= 0.0f && xp < v.res && yp >= 0.0f && yp < v.res && depth > 0.0f;
    float fx = __fsub_rn(__fdiv_rn(__fmul_rn(__fadd_rn(xp, 0.5f), static_cast<float>(v.w)), v.res), 0.5f);
    float fy = __fsub_rn(__fdiv_rn(__fmul_rn(__fadd_rn(yp, 0.5f), static_cast<float>(v.h)), v.res), 0.5f);
    fx = clamp_ref(fx, static_cast<float>(v.w - 1));
    fy = clamp_ref(fy, static_cast<float>(v.h - 1));
    c.x0 = static_cast<int>(floorf(fx));
    const int y0 = static_cast<int>(floorf(fy));
    c.x1 = min(c.x0 + 1, v.w - 1);
    const int y1 = min(y0 + 1, v.h - 1);
    c.wx = __fsub_rn(fx, static_cast<float>(c.x0));
    c.wy = __fsub_rn(fy, static_cast<float>(y0));
    c.top = static_cast<int64_t>(y0) * v.w;
    c.bottom = static_cast<int64_t>(y1) * v.w;
    return c;
}

__device__ __forceinline__ float lerp2(float tl, float tr, float bl, float br, float wx, float wy) {
    const float omx = __fsub_rn(1.0f, wx), omy = __fsub_rn(1.0f, wy);
    const float top = __fadd_rn(__fmul_rn(tl, omx), __fmul_rn(tr, wx));
    const float bot = __fadd_rn(__fmul_rn(bl, omx), __fmul_rn(br, wx));
    return __fadd_rn(__fmul_rn(top, omy), __fmul_rn(bot, wy));
}

template <typename TO>
__device__ __forceinline__ void store4(TO *o, float a, float b, float c, float d);
template <>
__device__ __forceinline__ void store4<float>(float *o, float a, float b, float c, float d) {
    *reinterpret_cast<float4 *>(o) = make_float4(a, b, c, d);
}
template <>
__device__ __forceinline__ void store4<__half>(__half *o, float a, float b, float c, float d) {
    uint2 u;
    u.x = pack2<__half>(a, b);
    u.y = pack2<__half>(c, d);
    *reinterpret_cast<uint2 *>(o) = u;
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16 *o, float a, float b, float c, float d) {
    uint2 u;
    u.x = pack2<__nv_bfloat16>(a, b);
    u.y = pack2<__nv_bfloat16>(c, d);
    *reinterpret_cast<uint2 *>(o) = u;
}

// VEC = 4: channels % 4 == 0, maps and output rows aligned for 16-byte
// loads and 4-element stores; VEC = 1: one channel per lane.
template <typename TO, int VEC>
__global__ void __launch_bounds__(32 * kProjWarps) project_kernel(const __grid_constant__ ProjParams p) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kProjWarps;
    const int r = p.grid;
    const int C = p.channels;
    for (int64_t pt = static_cast<int64_t>(blockIdx.x) * kProjWarps + (threadIdx.x >> 5); pt < p.n; pt += warps) {
        int ix, iy, iz;
        bool bad = false;
        if (p.coords) {
            const int4 c = reinterpret_cast<const int4 *>(p.coords)[pt];
            bad = c.x != 0 || c.y < 0 || c.z < 0 || c.w < 0 || c.y >= r || c.z >= r || c.w >= r;
            ix = c.y, iy = c.z, iz = c.w;
        } else {
            ix = static_cast<int>(pt / (static_cast<int64_t>(r) * r));
            iy = static_cast<int>((pt / r) % r);
            iz = static_cast<int>(pt % r);
        }
        TO *orow = reinterpret_cast<TO *>(p.out) + pt * p.ldo;
        if (bad) {  // warp-uniform
            if (lane == 0) latch_fault(p.fault, P3D_ERR_INVALID);
            for (int c = lane; c < C; c += 32) orow[c] = from_f32<TO>(0.0f);
            if (p.valid && lane == 0) p.valid[pt] = 0;
            continue;
        }
        const float bx = grid_base(ix, r), by = grid_base(iy, r), bz = grid_base(iz, r);
        Corner g{};
        if (lane < p.nviews) g = view_geometry(p.view[lane], bx, by, bz);
        const unsigned any_valid = __ballot_sync(0xffffffffu, lane < p.nviews && g.valid);
        if (p.valid && lane == 0) p.valid[pt] = any_valid ? 1 : 0;
        for (int c0 = 0; c0 < C; c0 += 32 * VEC) {
            const int c = c0 + lane * VEC;
            float acc[VEC];
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[e] = 0.0f;
            for (int v = 0; v < p.nviews; ++v) {
                const int64_t top = __shfl_sync(0xffffffffu, g.top, v);
                const int64_t bottom = __shfl_sync(0xffffffffu, g.bottom, v);
                const int x0 = __shfl_sync(0xffffffffu, g.x0, v);
                const int x1 = __shfl_sync(0xffffffffu, g.x1, v);
                const float wx = __shfl_sync(0xffffffffu, g.wx, v);
                const float wy = __shfl_sync(0xffffffffu, g.wy, v);
                if (c >= C) continue;
                const float *f = p.view[v].fmap;
                const int64_t tl = (top + x0) * C + c, tr = (top + x1) * C + c;
                const int64_t bl = (bottom + x0) * C + c, br = (bottom + x1) * C + c;
                if (VEC == 4) {
                    const float4 a = __ldg(reinterpret_cast<const float4 *>(f + tl));
                    const float4 b = __ldg(reinterpret_cast<const float4 *>(f + tr));
                    const float4 d = __ldg(reinterpret_cast<const float4 *>(f + bl));
                    const float4 e = __ldg(reinterpret_cast<const float4 *>(f + br));
                    const float s[4] = {lerp2(a.x, b.x, d.x, e.x, wx, wy), lerp2(a.y, b.y, d.y, e.y, wx, wy),
                                        lerp2(a.z, b.z, d.z, e.z, wx, wy), lerp2(a.w, b.w, d.w, e.w, wx, wy)};
#pragma unroll
                    for (int k = 0; k < VEC; ++k) acc[k] = p.nviews == 1 ? s[k] : __fadd_rn(acc[k], s[k]);
                } else {
                    const float s = lerp2(__ldg(f + tl), __ldg(f + tr), __ldg(f + bl), __ldg(f + br), wx, wy);
                    acc[0] = p.nviews == 1 ? s : __fadd_rn(acc[0], s);
                }
            }
            if (c >= C) continue;
            if (p.nviews > 1) {
#pragma unroll
                for (int k = 0; k < VEC; ++k) acc[k] = __fmul_rn(acc[k], p.inv_views);
            }
            if (VEC == 4)
                store4<TO>(orow + c, acc[0], acc[1], acc[2], acc[VEC - 1]);
            else
                orow[c] = from_f32<TO>(acc[0]);
        }
    }
}

// Gauss-Jordan inverse with partial pivoting on [M | I] in f32 (the
// reference's invert4x4, src/projection.cpp:47-98: first row of largest
// |pivot| wins, rows scaled by the pivot, eliminated in row order), so the
// world-to-camera matrix is the same to the last bit.
bool invert4(const float *in, float *out) {
    float a[4][8] = {};
    for (int r = 0; r < 4; ++r) {
        for (int c = 0; c < 4; ++c) a[r][c] = in[r * 4 + c];
        a[r][r + 4] = 1.0f;
    }
    for (int col = 0; col < 4; ++col) {
        int piv = col;
        float best = std::fabs(a[col][col]);
        for (int row = col + 1; row < 4; ++row)
            if (std::fabs(a[row][col]) > best) piv = row, best = std::fabs(a[row][col]);
        if (!(best > 1e-8f) || !std::isfinite(best)) return false;
        if (piv != col)
            for (int c = 0; c < 8; ++c) std::swap(a[piv][c], a[col][c]);
        const float s = a[col][col];
        for (int c = 0; c < 8; ++c) a[col][c] /= s;
        for (int row = 0; row < 4; ++row) {
            if (row == col) continue;
            const float f = a[row][col];
            if (f == 0.0f) continue;
            for (int c = 0; c < 8; ++c) a[row][c] -= f * a[col][c];
        }
    }
    for (int r = 0; r < 4; ++r)
        for (int c = 0; c < 4; ++c) out[r * 4 + c] = a[r][c + 4];
    return true;
}

void front_matrix(float distance, float *m) {
    const float f[16] = {1, 0, 0, 0, 0, 0, -1, -distance, 0, 1, 0, 0, 0, 0, 0, 1};
    for (int i = 0; i < 16; ++i) m[i] = f[i];
}

void mul4(const float *a, const float *b, float *out) {
    for (int r = 0; r < 4; ++r)
        for (int c = 0; c < 4; ++c) {
            float v = 0.0f;
            for (int k = 0; k < 4; ++k) v += a[r * 4 + k] * b[k * 4 + c];
            out[r * 4 + c] = v;
        }
}

// prepare_projection_view + validate_options (src/projection.cpp:205-259),
// with the reference's messages.
int view_constants(p3d_ctx *ctx, const p3d_projection_view &v, int grid, ViewConst &k) {
    constexpr float kPi = 3.14159265358979323846f;
    if (!v.feature_map) return set_error(ctx, P3D_ERR_INVALID, "feature_map is null");
    if (v.height <= 0 || v.width <= 0 || v.channels <= 0)
        return set_error(ctx, P3D_ERR_INVALID, "feature map dimensions must be positive");
    if (grid <= 0) return set_error(ctx, P3D_ERR_INVALID, "grid_resolution must be positive");
    if (v.image_resolution <= 0) return set_error(ctx, P3D_ERR_INVALID, "image_resolution must be positive");
    if (!(v.camera_angle_x > 0.0f && v.camera_angle_x < kPi) || !std::isfinite(v.camera_angle_x))
        return set_error(ctx, P3D_ERR_INVALID, "camera_angle_x must be finite and in (0, pi)");
    if (!(v.mesh_scale > 0.0f) || !std::isfinite(v.mesh_scale))
        return set_error(ctx, P3D_ERR_INVALID, "mesh_scale must be finite and positive");
    if (!v.has_transform && (!(v.distance > 0.0f) || !std::isfinite(v.distance)))
        return set_error(ctx, P3D_ERR_INVALID, "distance must be finite and positive");
    float c2w[16], w2c[16];
    if (v.has_transform)
        for (int i = 0; i < 16; ++i) c2w[i] = v.transform_matrix[i];
    else
        front_matrix(v.distance, c2w);
    if (!invert4(c2w, w2c)) return set_error(ctx, P3D_ERR_INVALID, "camera transform matrix is singular");
    k.fmap = v.feature_map;
    k.h = v.height;
    k.w = v.width;
    for (int i = 0; i < 12; ++i) k.w2c[i] = w2c[i];
    k.scale = 1.0f / (v.mesh_scale * 2.0f);
    const float focal = 16.0f / std::tan(v.camera_angle_x * 0.5f);
    k.focal_px = focal * static_cast<float>(v.image_resolution) / 32.0f;
    k.half = static_cast<float>(v.image_resolution) * 0.5f;
    k.res = static_cast<float>(v.image_resolution);
    return P3D_OK;
}

}  // namespace
}  // namespace p3d

using namespace p3d;

extern "C" int p3d_project_features(p3d_ctx *ctx, const p3d_projection_view *views, int nviews, int grid_resolution,
                                    const int32_t *coords, int64_t n, void *out, int64_t ldo, int out_dtype,
                                    uint8_t *valid) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, views && nviews > 0, "at least one projection view is required");
    P3D_REQUIRE(ctx, nviews <= kMaxViews, "p3d_project_features: at most 8 views");
    P3D_REQUIRE(ctx, out_dtype == P3D_F32 || out_dtype == P3D_F16 || out_dtype == P3D_BF16,
                "p3d_project_features: bad out_dtype");
    ProjParams p{};
    for (int i = 0; i < nviews; ++i) {
        if (views[i].channels != views[0].channels)
            return set_error(ctx, P3D_ERR_INVALID, "all projection views must have the same channel count");
        int rc = view_constants(ctx, views[i], grid_resolution, p.view[i]);
        if (rc) return rc;
    }
    const int C = views[0].channels;
    P3D_REQUIRE(ctx, n >= 0 && (n == 0 || (out && ldo >= C)), "p3d_project_features: bad output");
    if (n == 0) return P3D_OK;
    if (!coords) {
        const int64_t r = grid_resolution;
        P3D_REQUIRE(ctx, r <= 2048 && n == r * r * r, "p3d_project_features: dense grid needs n == grid^3");
    } else {
        P3D_REQUIRE(ctx, (reinterpret_cast<uintptr_t>(coords) & 15) == 0,
                    "p3d_project_features: coords must be 16-byte aligned");
    }
    p.nviews = nviews;
    p.grid = grid_resolution;
    p.channels = C;
    p.out_dtype = out_dtype;
    p.coords = coords;
    p.n = n;
    p.ldo = ldo;
    p.out = out;
    p.valid = valid;
    p.inv_views = 1.0f / static_cast<float>(nviews);
    p.fault = ctx->fault;
    const int64_t es = out_dtype == P3D_F32 ? 4 : 2;
    bool vec = C % 4 == 0 && (reinterpret_cast<uintptr_t>(out) % (4 * es)) == 0 && (ldo * es) % (4 * es) == 0;
    for (int i = 0; i < nviews; ++i) vec = vec && (reinterpret_cast<uintptr_t>(views[i].feature_map) & 15) == 0;
    DeviceGuard guard(ctx->device);
    const int64_t blocks64 = std::min<int64_t>((n + kProjWarps - 1) / kProjWarps, int64_t(ctx->num_sms) * 16);
    const dim3 grid(static_cast<unsigned>(blocks64)), block(32 * kProjWarps);
#define P3D_PROJ_LAUNCH(TO)                                                   \
    do {                                                                      \
        if (vec)                                                              \
            project_kernel<TO, 4><<<grid, block, 0, ctx->stream>>>(p);        \
        else                                                                  \
            project_kernel<TO, 1><<<grid, block, 0, ctx->stream>>>(p);        \
    } while (0)
    if (out_dtype == P3D_F32)
        P3D_PROJ_LAUNCH(float);
    else if (out_dtype == P3D_F16)
        P3D_PROJ_LAUNCH(__half);
    else
        P3D_PROJ_LAUNCH(__nv_bfloat16);
#undef P3D_PROJ_LAUNCH
    return check_launch(ctx, "project_features");
}

extern "C" int p3d_projection_relative_matrices(p3d_ctx *ctx, const float *c2w, const float *distances, int nviews,
                                                float *relative) {
    // ctx only carries the message (may be NULL: host math, no device work)
    auto fail = [ctx](const char *msg) { return ctx ? set_error(ctx, P3D_ERR_INVALID, msg) : int(P3D_ERR_INVALID); };
    if (!c2w || !distances || !relative || nviews <= 0) return fail("at least one camera transform is required");
    if (!(distances[0] > 0.0f) || !std::isfinite(distances[0]))
        return fail("main-view distance must be finite and positive");
    float inv[16], front[16], tmp[16];
    if (!invert4(c2w, inv)) return fail("main-view camera transform matrix is singular");
    front_matrix(distances[0], front);
    for (int i = 0; i < nviews; ++i) {
        mul4(inv, c2w + 16 * i, tmp);
        mul4(front, tmp, relative + 16 * i);
    }
    return P3D_OK;
}
