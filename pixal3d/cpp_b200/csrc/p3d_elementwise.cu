// Fused, vectorised elementwise / normalisation kernels of the SLat block:
// LayerNorm (+affine) (+AdaLN modulate), per-head RMS norm + 3D RoPE,
// activations, GroupNorm (+SiLU), and the Euler/CFG flow update.
// All are HBM-bound: one read and one write of each row, f32 math.
#include <algorithm>

#include "p3d_common.cuh"

namespace p3d {
namespace {

unsigned blocks_for(int64_t n, int per_block) { return static_cast<unsigned>(ceil_div(n, per_block)); }

template <typename T>
__device__ __forceinline__ void store_val(T *p, float v) {
    *p = from_f32<T>(v);
}

// ------------------------------------------------------------- LayerNorm
// One warp per row.  Two-pass statistics like sparse_layer_norm
// (src/sparse.cpp:514-531): mean, then mean of squared deviations.
template <typename TO, bool VEC>
__global__ void layernorm_mod_kernel(const float *__restrict__ x, int64_t n, int C, float eps,
                                     const float *__restrict__ gamma, const float *__restrict__ beta,
                                     const float *__restrict__ mod, int64_t mod_ld,
                                     const int32_t *__restrict__ offsets, int nbatch, TO *__restrict__ out) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n) return;
    const int lane = threadIdx.x & 31;
    const float *xr = x + row * C;
    float s = 0.0f;
    if (VEC) {
        for (int c = lane * 4; c < C; c += 128) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + c);
            s += (v.x + v.y) + (v.z + v.w);
        }
    } else {
        for (int c = lane; c < C; c += 32) s += xr[c];
    }
    const float mean = warp_sum(s) / static_cast<float>(C);
    float ss = 0.0f;
    if (VEC) {
        for (int c = lane * 4; c < C; c += 128) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + c);
            const float a = v.x - mean, b = v.y - mean, cc = v.z - mean, d = v.w - mean;
            ss += (a * a + b * b) + (cc * cc + d * d);
        }
    } else {
        for (int c = lane; c < C; c += 32) {
            const float d = xr[c] - mean;
            ss += d * d;
        }
    }
    const float var = warp_sum(ss) / static_cast<float>(C);
    const float inv = 1.0f / sqrtf(var + eps);
    const float *shift = nullptr, *scale = nullptr;
    if (mod) {
        const int b = batch_of_row(offsets, nbatch, row);
        shift = mod + static_cast<int64_t>(b) * mod_ld;
        scale = shift + C;
    }
    TO *o = out + row * C;
    for (int c = lane; c < C; c += 32) {
        float v = (xr[c] - mean) * inv;
        if (gamma) v = v * gamma[c] + beta[c];
        if (mod) v = v * (1.0f + scale[c]) + shift[c];
        store_val(o + c, v);
    }
}

// Register-resident variant for C = 128*NV: each lane holds its NV float4
// slices of the row, so x is read from HBM once; the same two-pass
// statistics, vectorised 16-byte parameter loads and 8/16-byte stores.
template <typename TO>
__device__ __forceinline__ void store4(TO *p, float a, float b, float c, float d) {
    if constexpr (sizeof(TO) == 4) {
        *reinterpret_cast<float4 *>(p) = make_float4(a, b, c, d);
    } else {
        *reinterpret_cast<uint2 *>(p) = make_uint2(pack2<TO>(a, b), pack2<TO>(c, d));
    }
}

// C = 1024 (NV = 8, the trunk): 4 blocks per SM (64 registers) keep 4,736
// rows in flight instead of 3,552 at the unbounded 74 registers (8,184 x 1,024
// f32 -> f16 with modulation: 9.84 -> 8.48 us).
template <typename TO, int NV>
__global__ void __launch_bounds__(256, NV == 8 ? 4 : 1) layernorm_reg_kernel(const float *__restrict__ x, int64_t n, float eps,
                                                            const float *__restrict__ gamma,
                                                            const float *__restrict__ beta,
                                                            const float *__restrict__ mod, int64_t mod_ld,
                                                            const int32_t *__restrict__ offsets, int nbatch,
                                                            TO *__restrict__ out) {
    constexpr int C = 128 * NV;
    pdl_wait();
    pdl_trigger();
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n) return;
    const int lane = threadIdx.x & 31;
    const float4 *xr = reinterpret_cast<const float4 *>(x + row * C);
    float4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = __ldcs(xr + i * 32 + lane);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    const float mean = warp_sum(s) / static_cast<float>(C);
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        v[i].x -= mean;
        v[i].y -= mean;
        v[i].z -= mean;
        v[i].w -= mean;
        ss += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
    }
    const float inv = 1.0f / sqrtf(warp_sum(ss) / static_cast<float>(C) + eps);
    const float4 *shift = nullptr, *scale = nullptr;
    if (mod) {
        const int b = batch_of_row(offsets, nbatch, row);
        shift = reinterpret_cast<const float4 *>(mod + static_cast<int64_t>(b) * mod_ld);
        scale = shift + C / 4;
    }
    TO *o = out + row * C;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c4 = i * 32 + lane;
        float4 y = make_float4(v[i].x * inv, v[i].y * inv, v[i].z * inv, v[i].w * inv);
        if (gamma) {
            const float4 g = __ldg(reinterpret_cast<const float4 *>(gamma) + c4);
            const float4 bb = __ldg(reinterpret_cast<const float4 *>(beta) + c4);
            y = make_float4(y.x * g.x + bb.x, y.y * g.y + bb.y, y.z * g.z + bb.z, y.w * g.w + bb.w);
        }
        if (mod) {
            const float4 sc = __ldg(scale + c4), sh = __ldg(shift + c4);
            y = make_float4(y.x * (1.0f + sc.x) + sh.x, y.y * (1.0f + sc.y) + sh.y, y.z * (1.0f + sc.z) + sh.z,
                            y.w * (1.0f + sc.w) + sh.w);
        }
        store4(o + 4 * c4, y.x, y.y, y.z, y.w);
    }
}

// LayerNorm (+affine) (+SiLU) into an operand of row pitch ld_out >= C whose
// pitch padding is written as zeros.  One warp per row, two-pass statistics
// (sparse_layer_norm, src/sparse.cpp:514-531).
template <typename TO>
__global__ void layernorm_act_kernel(const float *__restrict__ x, int64_t n, int C, float eps,
                                     const float *__restrict__ gamma, const float *__restrict__ beta, int silu,
                                     TO *__restrict__ out, int64_t ld_out) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n) return;
    const int lane = threadIdx.x & 31;
    const float *xr = x + row * C;
    float s = 0.0f;
    for (int c = lane; c < C; c += 32) s += xr[c];
    const float mean = warp_sum(s) / static_cast<float>(C);
    float ss = 0.0f;
    for (int c = lane; c < C; c += 32) {
        const float d = xr[c] - mean;
        ss += d * d;
    }
    const float inv = 1.0f / sqrtf(warp_sum(ss) / static_cast<float>(C) + eps);
    TO *o = out + row * ld_out;
    for (int c = lane; c < ld_out; c += 32) {
        float v = 0.0f;
        if (c < C) {
            v = (xr[c] - mean) * inv;
            if (gamma) v = v * gamma[c] + beta[c];
            if (silu) v = silu_f(v);
        }
        store_val(o + c, v);
    }
}

// f32 [rows][cols] -> TO [rows][ld] with zero pitch padding.
template <typename TO>
__global__ void pack_operand_kernel(const float *__restrict__ x, int64_t rows, int cols, TO *__restrict__ out,
                                    int64_t ld) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= rows * ld) return;
    const int64_t r = i / ld;
    const int64_t c = i - r * ld;
    store_val(out + i, c < cols ? x[r * cols + c] : 0.0f);
}

// ------------------------------------------------ per-head RMS + 3D RoPE
// One warp per row; lane p owns rotation pair p (elements 2p, 2p+1) of
// every head.  head_dim <= 64.
template <typename T>
__global__ void qk_rms_rope_kernel(T *__restrict__ x, int64_t n, int64_t ld, int heads, int hd,
                                   const float *__restrict__ gamma, const int4 *__restrict__ coords, float fmin,
                                   float fbase) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n) return;
    const int lane = threadIdx.x & 31;
    const int pairs = hd / 2;
    const bool active = lane < pairs;
    float cs = 1.0f, sn = 0.0f;
    if (coords && active) {
        const int fd = pairs / 3;
        if (lane < 3 * fd) {
            const int4 c = coords[row];
            const int axis = lane / fd;
            const int coord = axis == 0 ? c.y : (axis == 1 ? c.z : c.w);
            const float freq = fmin / powf(fbase, static_cast<float>(lane % fd) / static_cast<float>(fd));
            const float phase = static_cast<float>(coord) * freq;
            sincosf(phase, &sn, &cs);
        }
    }
    const float mult = sqrtf(static_cast<float>(hd));
    T *xr = x + row * ld;
    for (int h = 0; h < heads; ++h) {
        float e = 0.0f, o = 0.0f;
        uint32_t *pp = reinterpret_cast<uint32_t *>(xr + h * hd + 2 * lane);
        if (active) {
            const float2 v = unpack2<T>(*pp);
            e = v.x;
            o = v.y;
        }
        if (gamma) {
            const float sq = warp_sum(e * e + o * o);
            const float inv = 1.0f / fmaxf(sqrtf(sq), 1e-12f);
            if (active) {
                e = e * inv * mult * gamma[h * hd + 2 * lane];
                o = o * inv * mult * gamma[h * hd + 2 * lane + 1];
            }
        }
        if (active) {
            const float re = e * cs - o * sn;
            const float ro = e * sn + o * cs;
            *pp = pack2<T>(re, ro);
        }
    }
}

// One thread per (pair, point): the cos/sin that qk_rms_rope_kernel computes
// on the fly, stored once per coordinate set, pair-major (table[pr][row]).
__global__ void rope_table_kernel(const int4 *__restrict__ coords, int64_t n, int pairs, float fmin, float fbase,
                                  float2 *__restrict__ table) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n * pairs) return;
    const int pr = static_cast<int>(i / n);
    const int64_t row = i - static_cast<int64_t>(pr) * n;
    const int fd = pairs / 3;
    float cs = 1.0f, sn = 0.0f;
    if (pr < 3 * fd) {
        const int4 c = coords[row];
        const int axis = pr / fd;
        const int coord = axis == 0 ? c.y : (axis == 1 ? c.z : c.w);
        const float freq = fmin / powf(fbase, static_cast<float>(pr % fd) / static_cast<float>(fd));
        sincosf(static_cast<float>(coord) * freq, &sn, &cs);
    }
    table[i] = make_float2(cs, sn);
}

// out[row][h][c] = c < hd_in ? x[row][h][c] : 0 for c < hd_out, and the
// row's pitch padding [heads*hd_out, ldo) = 0: moves heads between head
// widths (e.g. head_dim 6 <-> the attention kernel's 64).
template <typename T>
__global__ void repack_heads_kernel(const T *__restrict__ x, int64_t ldx, int64_t n, int heads, int hd_in,
                                    int hd_out, T *__restrict__ out, int64_t ldo) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n * ldo) return;
    const int64_t row = i / ldo;
    const int64_t r = i - row * ldo;
    T v = from_f32<T>(0.0f);
    if (r < static_cast<int64_t>(heads) * hd_out) {
        const int h = static_cast<int>(r / hd_out), c = static_cast<int>(r - static_cast<int64_t>(h) * hd_out);
        if (c < hd_in) v = x[row * ldx + static_cast<int64_t>(h) * hd_in + c];
    }
    out[i] = v;
}

// ------------------------------------------------------------ activations
template <typename T>
__global__ void activation_kernel(const T *__restrict__ x, int64_t n, int act, T *__restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = to_f32(x[i]);
    store_val(out + i, act == P3D_EPI_GELU_TANH ? gelu_tanh_f(v) : silu_f(v));
}

// ------------------------------------------------------------- GroupNorm
// Stats, generic layout: each block walks a contiguous row range with one
// float4 per thread per row step (C/4 threads span a row, coalesced),
// accumulating per element e of the float4 the sum and sum of squares of its
// group (4*cb + e) / gs in double (a float4 may span several groups when the
// group is narrower than 4 channels); one atomicAdd per element and group
// whenever the batch item changes or the range ends.  Requires C % 4 == 0.
__global__ void groupnorm_stats_kernel(const float *__restrict__ x, int64_t n, int C, int groups,
                                       const int32_t *__restrict__ offsets, int nbatch, int rows_per_block,
                                       double *__restrict__ stats) {
    const int c4 = C / 4;
    const int tpr = blockDim.x < c4 ? blockDim.x : c4;  // threads per row
    const int rows_step = blockDim.x / tpr;
    const int t = threadIdx.x;
    const int col4 = t % tpr, rsub = t / tpr;
    if (rsub >= rows_step) return;  // blockDim not a multiple of tpr: spare threads
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
    const int64_t r1 = min(n, r0 + rows_per_block);
    const int gs = C / groups;
    for (int cb = col4; cb < c4; cb += tpr) {
        int g[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) g[e] = (4 * cb + e) / gs;
        double sum[4] = {0.0, 0.0, 0.0, 0.0}, sq[4] = {0.0, 0.0, 0.0, 0.0};
        int cur_b = -1;
        auto flush = [&](int b) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (sum[e] != 0.0 || sq[e] != 0.0) {
                    atomicAdd(stats + 2 * (b * groups + g[e]), sum[e]);
                    atomicAdd(stats + 2 * (b * groups + g[e]) + 1, sq[e]);
                }
                sum[e] = sq[e] = 0.0;
            }
        };
        for (int64_t r = r0 + rsub; r < r1; r += rows_step) {
            const int b = batch_of_row(offsets, nbatch, r);
            if (b != cur_b) {
                if (cur_b >= 0) flush(cur_b);
                cur_b = b;
            }
            const float4 v = __ldg(reinterpret_cast<const float4 *>(x + r * C) + cb);
            const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                sum[e] += static_cast<double>(vv[e]);
                sq[e] += static_cast<double>(vv[e]) * vv[e];
            }
        }
        if (cur_b >= 0) flush(cur_b);
    }
}

// Stats, rows layout (C = 128 * NV): a block owns a contiguous row range,
// split at batch-item boundaries; each warp reads whole rows (lane l holds
// float4 l + 32j, j < NV: every load instruction covers 512 contiguous bytes,
// NV loads in flight per lane) and keeps per-j f32 partial sums over its few
// rows (a handful of rows x 4 channels per lane).  Lanes sharing a group are
// combined in double by shuffles when the group is a power-of-two number of
// float4 wide (or a multiple of 128 channels), then per block in shared
// memory (double), then one global double atomic per group and batch segment.
template <int NV>
__global__ void __launch_bounds__(256, 3) groupnorm_stats_rows_kernel(const float *__restrict__ x, int64_t n,
                                                                     int groups, const int32_t *__restrict__ offsets,
                                                                     int nbatch, int64_t rows_per_block,
                                                                     double *__restrict__ stats) {
    extern __shared__ double gsum[];  // [2 * groups]
    constexpr int C = 128 * NV;
    const int gs = C / groups;
    const int w = gs >> 2;  // lanes per group within one 128-channel block
    const int mode = (gs % 128 == 0) ? 2 : ((w & (w - 1)) == 0 ? 1 : 0);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
    const int64_t r1 = min(n, r0 + rows_per_block);
    for (int i = threadIdx.x; i < 2 * groups; i += blockDim.x) gsum[i] = 0.0;
    __syncthreads();
    for (int b = 0; b < nbatch; ++b) {
        const int64_t s0 = max(r0, static_cast<int64_t>(offsets[b]));
        const int64_t s1 = min(r1, static_cast<int64_t>(offsets[b + 1]));
        if (s0 >= s1) continue;  // block-uniform
        float sum[NV], sq[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) sum[j] = sq[j] = 0.0f;
        for (int64_t r = s0 + warp; r < s1; r += nwarps) {
            const float4 *xr = reinterpret_cast<const float4 *>(x + r * C) + lane;
            float4 v[NV];
#pragma unroll
            for (int j = 0; j < NV; ++j) v[j] = __ldg(xr + 32 * j);
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                sum[j] += (v[j].x + v[j].y) + (v[j].z + v[j].w);
                sq[j] += (v[j].x * v[j].x + v[j].y * v[j].y) + (v[j].z * v[j].z + v[j].w * v[j].w);
            }
        }
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            double su = sum[j], qu = sq[j];
            const int g = (128 * j + 4 * lane) / gs;
            if (mode == 2) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    su += __shfl_xor_sync(0xffffffffu, su, o);
                    qu += __shfl_xor_sync(0xffffffffu, qu, o);
                }
                if (lane == 0) {
                    atomicAdd(&gsum[2 * g], su);
                    atomicAdd(&gsum[2 * g + 1], qu);
                }
            } else if (mode == 1) {
                for (int o = 1; o < w; o <<= 1) {
                    su += __shfl_xor_sync(0xffffffffu, su, o);
                    qu += __shfl_xor_sync(0xffffffffu, qu, o);
                }
                if ((lane & (w - 1)) == 0) {
                    atomicAdd(&gsum[2 * g], su);
                    atomicAdd(&gsum[2 * g + 1], qu);
                }
            } else {
                atomicAdd(&gsum[2 * g], su);
                atomicAdd(&gsum[2 * g + 1], qu);
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < 2 * groups; i += blockDim.x) {
            if (gsum[i] != 0.0) atomicAdd(stats + 2 * b * groups + i, gsum[i]);
            gsum[i] = 0.0;
        }
        __syncthreads();
    }
}

// mean / rstd per (batch, group) from the double sums.
__global__ void groupnorm_finalize_kernel(const double *__restrict__ stats, const int32_t *__restrict__ offsets,
                                          int nbatch, int groups, int C, float eps, float *__restrict__ mr) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nbatch * groups) return;
    const int b = i / groups;
    const double cnt = static_cast<double>(offsets[b + 1] - offsets[b]) * (C / groups);
    const double mean = cnt > 0 ? stats[2 * i] / cnt : 0.0;
    const double var = cnt > 0 ? fmax(stats[2 * i + 1] / cnt - mean * mean, 0.0) : 0.0;
    mr[2 * i] = static_cast<float>(mean);
    mr[2 * i + 1] = static_cast<float>(1.0 / sqrt(var + static_cast<double>(eps)));
}

// Apply, rows layout (C = 128 * NV): a warp per row (grid-stride), lane l
// holds float4 l + 32j as in the stats kernel, so neither a row index
// division nor a per-element batch search is needed; all NV loads of a row
// are issued before its math.
template <int NV, typename TO>
__global__ void __launch_bounds__(256, 3) groupnorm_apply_rows_kernel(const float *__restrict__ x, int64_t n,
                                                                      int groups, const float *__restrict__ gamma,
                                                                      const float *__restrict__ beta,
                                                                      const int32_t *__restrict__ offsets, int nbatch,
                                                                      const float *__restrict__ mr, int silu,
                                                                      TO *__restrict__ out) {
    constexpr int C = 128 * NV;
    const int gs = C / groups;
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n; r += warps) {
        const float4 *xr = reinterpret_cast<const float4 *>(x + r * C) + lane;
        float4 v[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) v[j] = __ldg(xr + 32 * j);
        const float *mrb = mr + 2 * batch_of_row(offsets, nbatch, r) * groups;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int cb = lane + 32 * j;  // float4 index within the row
            const int g = (cb * 4) / gs;
            const float mean = __ldg(mrb + 2 * g), rstd = __ldg(mrb + 2 * g + 1);
            float y[4] = {(v[j].x - mean) * rstd, (v[j].y - mean) * rstd, (v[j].z - mean) * rstd,
                          (v[j].w - mean) * rstd};
            if (gamma) {
                const float4 ga = __ldg(reinterpret_cast<const float4 *>(gamma) + cb);
                const float4 be = __ldg(reinterpret_cast<const float4 *>(beta) + cb);
                y[0] = y[0] * ga.x + be.x;
                y[1] = y[1] * ga.y + be.y;
                y[2] = y[2] * ga.z + be.z;
                y[3] = y[3] * ga.w + be.w;
            }
            if (silu) {
#pragma unroll
                for (int e = 0; e < 4; ++e) y[e] = silu_f(y[e]);
            }
            TO *o = out + r * C + cb * 4;
            if constexpr (sizeof(TO) == 2) {
                uint2 pk;
                pk.x = pack2<TO>(y[0], y[1]);
                pk.y = pack2<TO>(y[2], y[3]);
                *reinterpret_cast<uint2 *>(o) = pk;
            } else {
                *reinterpret_cast<float4 *>(o) = make_float4(y[0], y[1], y[2], y[3]);
            }
        }
    }
}

// y = silu((x - mean) * rstd * gamma + beta).  Each thread handles 4 float4
// spaced blockDim apart (coalesced), all 4 loads issued before any math.
constexpr int kGnApplyVec = 4;
template <typename TO>
__global__ void __launch_bounds__(256) groupnorm_apply_kernel(const float *__restrict__ x, int64_t n, int C,
                                                              int groups, const float *__restrict__ gamma,
                                                              const float *__restrict__ beta,
                                                              const int32_t *__restrict__ offsets, int nbatch,
                                                              const float *__restrict__ mr, int silu,
                                                              TO *__restrict__ out) {
    const int c4 = C / 4;
    const int gs = C / groups;
    const int64_t total = n * c4;
    const int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x * kGnApplyVec + threadIdx.x;
    float4 v[kGnApplyVec];
#pragma unroll
    for (int k = 0; k < kGnApplyVec; ++k) {
        const int64_t i = base + static_cast<int64_t>(k) * blockDim.x;
        if (i < total) v[k] = __ldg(reinterpret_cast<const float4 *>(x) + i);
    }
#pragma unroll
    for (int k = 0; k < kGnApplyVec; ++k) {
        const int64_t i = base + static_cast<int64_t>(k) * blockDim.x;
        if (i >= total) break;
        const int64_t row = i / c4;
        const int cb = static_cast<int>(i - row * c4);
        const int b = batch_of_row(offsets, nbatch, row);
        const float vv[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
        float y[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {  // a float4 may span groups narrower than 4 channels
            const int g = (cb * 4 + e) / gs;
            y[e] = (vv[e] - __ldg(mr + 2 * (b * groups + g))) * __ldg(mr + 2 * (b * groups + g) + 1);
        }
        if (gamma) {
            const float4 ga = __ldg(reinterpret_cast<const float4 *>(gamma) + cb);
            const float4 be = __ldg(reinterpret_cast<const float4 *>(beta) + cb);
            y[0] = y[0] * ga.x + be.x;
            y[1] = y[1] * ga.y + be.y;
            y[2] = y[2] * ga.z + be.z;
            y[3] = y[3] * ga.w + be.w;
        }
        if (silu) {
#pragma unroll
            for (int e = 0; e < 4; ++e) y[e] = silu_f(y[e]);
        }
        TO *o = out + i * 4;
        if constexpr (sizeof(TO) == 2) {
            uint2 pk;
            pk.x = pack2<TO>(y[0], y[1]);
            pk.y = pack2<TO>(y[2], y[3]);
            *reinterpret_cast<uint2 *>(o) = pk;
        } else {
            *reinterpret_cast<float4 *>(o) = make_float4(y[0], y[1], y[2], y[3]);
        }
    }
}

// ------------------------------------------------------------ Euler / CFG
// x0 = a*x - b*v with a = 1 - sigma_min, b = sigma_min + a*t (pred_to_xstart,
// src/flow_sampler.cpp:139-147).  Stats per batch: sum/sumsq of x0(pos) and
// x0(cfg) for the guidance-rescale std (sparse_batch_std, :164-198).
__global__ void cfg_rescale_stats_kernel(const float *__restrict__ x, const float *__restrict__ vp,
                                         const float *__restrict__ vn, int64_t n, int C,
                                         const int32_t *__restrict__ offsets, int nbatch, float t, float g,
                                         float sigma_min, double *__restrict__ stats) {
    cfg_stats_rows(x, vp, vn, n, C, offsets, nbatch, t, g, sigma_min, stats);
}

__global__ void euler_cfg_kernel(float *__restrict__ x, const float *__restrict__ vp, const float *__restrict__ vn,
                                 int64_t n, int C, const int32_t *__restrict__ offsets, int nbatch, float t, float dt,
                                 float g, float gr, float sigma_min, const double *__restrict__ stats,
                                 float *__restrict__ x0_out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n * C) return;
    const float p = vp[i];
    float pred = vn ? g * p + (1.0f - g) * vn[i] : p;
    if (stats) {
        // apply_guidance_rescale (src/flow_sampler.cpp:210-241)
        const int64_t row = i / C;
        const int b = batch_of_row(offsets, nbatch, row);
        const double cnt = static_cast<double>(offsets[b + 1] - offsets[b]) * C;
        const double m0 = stats[4 * b] / cnt, m1 = stats[4 * b + 2] / cnt;
        const float sp = static_cast<float>(sqrt(fmax(stats[4 * b + 1] / cnt - m0 * m0, 0.0)));
        const float sc = static_cast<float>(sqrt(fmax(stats[4 * b + 3] / cnt - m1 * m1, 0.0)));
        const float ratio = sc != 0.0f ? sp / sc : 1.0f;
        const float a = 1.0f - sigma_min, bb = sigma_min + a * t;
        float x0 = a * x[i] - bb * pred;
        x0 = gr * (x0 * ratio) + (1.0f - gr) * x0;
        pred = (a * x[i] - x0) / bb;
    }
    if (x0_out) {
        // pred_to_xstart (src/flow_sampler.cpp:139-147) of the final prediction
        const float a = 1.0f - sigma_min, bb = sigma_min + a * t;
        x0_out[i] = a * x[i] - bb * pred;
    }
    x[i] -= dt * pred;
}

}  // namespace
}  // namespace p3d

using namespace p3d;

extern "C" int p3d_layernorm_modulate(p3d_ctx *ctx, const float *x, int64_t n, int channels, float eps,
                                      const float *gamma, const float *beta, const float *mod, int64_t mod_ld,
                                      const int32_t *batch_offsets, int nbatch, void *out, int out_dtype) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && out && channels > 0, "p3d_layernorm_modulate: bad argument");
    P3D_REQUIRE(ctx, (gamma == nullptr) == (beta == nullptr),
                "sparse layer norm affine parameters must be both null or non-null");
    P3D_REQUIRE(ctx, eps > 0.0f, "sparse layer norm epsilon must be finite and positive");
    P3D_REQUIRE(ctx, !mod || (batch_offsets && nbatch > 0), "p3d_layernorm_modulate: modulation needs batch offsets");
    if (n == 0) return P3D_OK;
    const bool vec = channels % 128 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const unsigned grid = blocks_for(n, 8);
    auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const int nv = channels / 128;
    const bool reg = vec && al16(out) && al16(gamma) && al16(beta) && al16(mod) && mod_ld % 4 == 0 &&
                     (nv == 1 || nv == 2 || nv == 3 || nv == 4 || nv == 6 || nv == 8 || nv == 12 || nv == 16);
    if (reg) {
#define P3D_LN_REG(NVV)                                                                                         \
    case NVV:                                                                                                  \
        P3D_CUDA(ctx, launch_pdl(layernorm_reg_kernel<TO, NVV>, dim3(grid), dim3(256), 0, ctx->stream, x, n, eps,   \
                                 gamma, beta, mod, mod_ld, batch_offsets, nbatch, static_cast<TO *>(out)));      \
        break;
        P3D_DISPATCH(out_dtype, TO, {
            switch (nv) {
                P3D_LN_REG(1) P3D_LN_REG(2) P3D_LN_REG(3) P3D_LN_REG(4) P3D_LN_REG(6) P3D_LN_REG(8) P3D_LN_REG(12)
                P3D_LN_REG(16)
            }
        });
#undef P3D_LN_REG
        return check_launch(ctx, "layernorm_mod");
    }
    P3D_DISPATCH(out_dtype, TO, {
        if (vec)
            layernorm_mod_kernel<TO, true><<<grid, 256, 0, ctx->stream>>>(
                x, n, channels, eps, gamma, beta, mod, mod_ld, batch_offsets, nbatch, static_cast<TO *>(out));
        else
            layernorm_mod_kernel<TO, false><<<grid, 256, 0, ctx->stream>>>(
                x, n, channels, eps, gamma, beta, mod, mod_ld, batch_offsets, nbatch, static_cast<TO *>(out));
    });
    return check_launch(ctx, "layernorm_mod");
}

extern "C" int p3d_layernorm_act(p3d_ctx *ctx, const float *x, int64_t n, int channels, float eps,
                                 const float *gamma, const float *beta, int silu, void *out, int64_t ld_out,
                                 int out_dtype) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && out && channels > 0 && ld_out >= channels && n >= 0, "p3d_layernorm_act: bad argument");
    P3D_REQUIRE(ctx, (gamma == nullptr) == (beta == nullptr),
                "sparse layer norm affine parameters must be both null or non-null");
    P3D_REQUIRE(ctx, eps > 0.0f, "sparse layer norm epsilon must be finite and positive");
    if (n == 0) return P3D_OK;
    P3D_DISPATCH(out_dtype, TO,
                 layernorm_act_kernel<TO><<<blocks_for(n, 8), 256, 0, ctx->stream>>>(
                     x, n, channels, eps, gamma, beta, silu, static_cast<TO *>(out), ld_out));
    return check_launch(ctx, "layernorm_act");
}

extern "C" int p3d_pack_operand(p3d_ctx *ctx, const float *x, int64_t rows, int cols, void *out, int64_t ld,
                                int out_dtype) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && out && cols > 0 && ld >= cols && rows >= 0, "p3d_pack_operand: bad argument");
    if (rows == 0) return P3D_OK;
    P3D_DISPATCH(out_dtype, TO,
                 pack_operand_kernel<TO><<<blocks_for(rows * ld, 256), 256, 0, ctx->stream>>>(
                     x, rows, cols, static_cast<TO *>(out), ld));
    return check_launch(ctx, "pack_operand");
}

extern "C" int p3d_qk_rmsnorm_rope(p3d_ctx *ctx, void *x, int64_t n, int64_t ld, int heads, int head_dim,
                                   const float *gamma, const int32_t *coords, float freq_min, float freq_base,
                                   int dtype) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && heads > 0 && head_dim > 0 && head_dim % 2 == 0 && head_dim <= 64,
                "sparse RoPE head dimensions are invalid");
    P3D_REQUIRE(ctx, ld >= static_cast<int64_t>(heads) * head_dim, "p3d_qk_rmsnorm_rope: ld too small");
    P3D_REQUIRE(ctx, (reinterpret_cast<uintptr_t>(x) & 3) == 0 && ld % 2 == 0, "p3d_qk_rmsnorm_rope: misaligned");
    P3D_REQUIRE(ctx, freq_min > 0.0f && freq_base > 0.0f, "sparse RoPE frequencies must be finite and positive");
    P3D_REQUIRE(ctx, is_16bit(dtype), "p3d_qk_rmsnorm_rope: dtype must be bf16 or f16");
    if (n == 0) return P3D_OK;
    if (dtype == P3D_BF16)
        qk_rms_rope_kernel<__nv_bfloat16><<<blocks_for(n, 8), 256, 0, ctx->stream>>>(
            static_cast<__nv_bfloat16 *>(x), n, ld, heads, head_dim, gamma, reinterpret_cast<const int4 *>(coords),
            freq_min, freq_base);
    else
        qk_rms_rope_kernel<__half><<<blocks_for(n, 8), 256, 0, ctx->stream>>>(
            static_cast<__half *>(x), n, ld, heads, head_dim, gamma, reinterpret_cast<const int4 *>(coords), freq_min,
            freq_base);
    return check_launch(ctx, "qk_rms_rope");
}

extern "C" int p3d_rope_table(p3d_ctx *ctx, const int32_t *coords, int64_t n, int head_dim, float freq_min,
                              float freq_base, float *table) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, coords && table && head_dim >= 2 && head_dim % 2 == 0 && n >= 0, "p3d_rope_table: bad argument");
    if (n == 0) return P3D_OK;
    const int pairs = head_dim / 2;
    rope_table_kernel<<<blocks_for(n * pairs, 256), 256, 0, ctx->stream>>>(
        reinterpret_cast<const int4 *>(coords), n, pairs, freq_min, freq_base, reinterpret_cast<float2 *>(table));
    return check_launch(ctx, "rope_table");
}

extern "C" int p3d_repack_heads(p3d_ctx *ctx, const void *x, int64_t ldx, int64_t n, int heads, int hd_in,
                                int hd_out, void *out, int64_t ldo, int dtype) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && out && x != out && heads > 0 && hd_in > 0 && hd_out > 0 && n >= 0,
                "p3d_repack_heads: bad argument");
    P3D_REQUIRE(ctx, ldx >= static_cast<int64_t>(heads) * hd_in && ldo >= static_cast<int64_t>(heads) * hd_out,
                "p3d_repack_heads: row pitch too small");
    const int64_t count = n * ldo;
    if (count == 0) return P3D_OK;
    P3D_DISPATCH(dtype, T,
                 repack_heads_kernel<T><<<blocks_for(count, 256), 256, 0, ctx->stream>>>(
                     static_cast<const T *>(x), ldx, n, heads, hd_in, hd_out, static_cast<T *>(out), ldo));
    return check_launch(ctx, "repack_heads");
}

extern "C" int p3d_activation(p3d_ctx *ctx, const void *x, int64_t count, int act, int dtype, void *out) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && out && (act == P3D_EPI_GELU_TANH || act == P3D_EPI_SILU), "p3d_activation: bad argument");
    if (count == 0) return P3D_OK;
    P3D_DISPATCH(dtype, T,
                 activation_kernel<T><<<blocks_for(count, 256), 256, 0, ctx->stream>>>(
                     static_cast<const T *>(x), count, act, static_cast<T *>(out)));
    return check_launch(ctx, "activation");
}

extern "C" int p3d_group_norm_silu(p3d_ctx *ctx, const float *x, int64_t n, int channels, int groups, float eps,
                                   const float *gamma, const float *beta, const int32_t *batch_offsets, int nbatch,
                                   int silu, double *stats, void *out, int out_dtype) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && out && stats && batch_offsets && nbatch > 0, "p3d_group_norm_silu: null pointer");
    P3D_REQUIRE(ctx, groups > 0 && channels % groups == 0 && channels % 4 == 0,
                "p3d_group_norm_silu: channels must be a multiple of 4 and of groups");
    P3D_REQUIRE(ctx, (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0,
                "p3d_group_norm_silu: x/out must be 16-byte aligned");
    P3D_REQUIRE(ctx, !gamma || (beta && (reinterpret_cast<uintptr_t>(gamma) & 15) == 0 &&
                                (reinterpret_cast<uintptr_t>(beta) & 15) == 0),
                "p3d_group_norm_silu: gamma/beta must be 16-byte aligned");
    // stats scratch: [nbatch*groups*2] double sums, then [nbatch*groups*2] float mean/rstd
    P3D_CUDA(ctx, cudaMemsetAsync(stats, 0, sizeof(double) * 2 * nbatch * groups, ctx->stream));
    if (n == 0) return P3D_OK;
    // Rows-layout kernels for C = 128 * NV (NV in 1, 2, 4, 8, 16) and groups of
    // whole float4s; the generic kernels take every other shape.
    const int nv = channels % 128 == 0 ? channels / 128 : 0;
    const bool rows = (nv == 1 || nv == 2 || nv == 4 || nv == 8 || nv == 16) && (channels / groups) % 4 == 0;
    if (rows) {
        // ~4 resident blocks per SM, each a contiguous row range
        const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 16), 4 * ctx->num_sms));
        const int64_t rpb = ceil_div(n, blocks);
        const unsigned grid = static_cast<unsigned>(ceil_div(n, rpb));
        const size_t sm = 2 * groups * sizeof(double);
        switch (nv) {
            case 1: groupnorm_stats_rows_kernel<1><<<grid, 256, sm, ctx->stream>>>(x, n, groups, batch_offsets, nbatch, rpb, stats); break;
            case 2: groupnorm_stats_rows_kernel<2><<<grid, 256, sm, ctx->stream>>>(x, n, groups, batch_offsets, nbatch, rpb, stats); break;
            case 4: groupnorm_stats_rows_kernel<4><<<grid, 256, sm, ctx->stream>>>(x, n, groups, batch_offsets, nbatch, rpb, stats); break;
            case 8: groupnorm_stats_rows_kernel<8><<<grid, 256, sm, ctx->stream>>>(x, n, groups, batch_offsets, nbatch, rpb, stats); break;
            default: groupnorm_stats_rows_kernel<16><<<grid, 256, sm, ctx->stream>>>(x, n, groups, batch_offsets, nbatch, rpb, stats); break;
        }
    } else {
        const int rows_per_block = 64;
        groupnorm_stats_kernel<<<blocks_for(n, rows_per_block), 256, 0, ctx->stream>>>(
            x, n, channels, groups, batch_offsets, nbatch, rows_per_block, stats);
    }
    int rc = check_launch(ctx, "groupnorm_stats");
    if (rc) return rc;
    float *mr = reinterpret_cast<float *>(stats + 2 * nbatch * groups);
    groupnorm_finalize_kernel<<<blocks_for(nbatch * groups, 128), 128, 0, ctx->stream>>>(
        stats, batch_offsets, nbatch, groups, channels, eps, mr);
    if ((rc = check_launch(ctx, "groupnorm_finalize"))) return rc;
    const int64_t count4 = n * (channels / 4);
    if (rows) {
        const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(n, 8), 16 * ctx->num_sms));
#define P3D_GN_APPLY(NV_)                                                                                      \
    P3D_DISPATCH(out_dtype, TO,                                                                                \
                 groupnorm_apply_rows_kernel<NV_, TO><<<grid, 256, 0, ctx->stream>>>(                          \
                     x, n, groups, gamma, beta, batch_offsets, nbatch, mr, silu, static_cast<TO *>(out)))
        switch (nv) {
            case 1: P3D_GN_APPLY(1); break;
            case 2: P3D_GN_APPLY(2); break;
            case 4: P3D_GN_APPLY(4); break;
            case 8: P3D_GN_APPLY(8); break;
            default: P3D_GN_APPLY(16); break;
        }
#undef P3D_GN_APPLY
        return check_launch(ctx, "groupnorm_apply");
    }
    P3D_DISPATCH(out_dtype, TO,
                 groupnorm_apply_kernel<TO><<<blocks_for(count4, 256 * kGnApplyVec), 256, 0, ctx->stream>>>(
                     x, n, channels, groups, gamma, beta, batch_offsets, nbatch, mr, silu, static_cast<TO *>(out)));
    return check_launch(ctx, "groupnorm_apply");
}

extern "C" int p3d_euler_cfg_step(p3d_ctx *ctx, float *x, const float *v_pos, const float *v_neg, int64_t n,
                                  int channels, const int32_t *batch_offsets, int nbatch, float t, float t_next,
                                  float guidance, float guidance_rescale, float sigma_min, double *stats, float *x0_out) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && v_pos && channels > 0, "p3d_euler_cfg_step: bad argument");
    const bool rescale = v_neg && guidance_rescale > 0.0f;
    P3D_REQUIRE(ctx, !rescale || (stats && batch_offsets && nbatch > 0),
                "p3d_euler_cfg_step: guidance rescale needs stats scratch and batch offsets");
    if (n == 0) return P3D_OK;
    if (rescale) {
        P3D_CUDA(ctx, cudaMemsetAsync(stats, 0, sizeof(double) * 4 * nbatch, ctx->stream));
        cfg_rescale_stats_kernel<<<blocks_for(ceil_div(n, kStatsRowsPerWarp), 8), 256, 0, ctx->stream>>>(
            x, v_pos, v_neg, n, channels,
                                                                          batch_offsets, nbatch, t, guidance,
                                                                          sigma_min, stats);
        int rc = check_launch(ctx, "cfg_rescale_stats");
        if (rc) return rc;
    }
    euler_cfg_kernel<<<blocks_for(n * channels, 256), 256, 0, ctx->stream>>>(
        x, v_pos, v_neg, n, channels, batch_offsets, nbatch, t, t - t_next, guidance, guidance_rescale, sigma_min,
        rescale ? stats : nullptr, x0_out);
    return check_launch(ctx, "euler_cfg");
}
