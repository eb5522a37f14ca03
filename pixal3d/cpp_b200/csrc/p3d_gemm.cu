// tcgen05/TMEM GEMM for the SLat hot path: dense linears and the
// gather-GEMM submanifold sparse convolution share one persistent,
// warp-specialised kernel.
//
//   C[m, n] = epilogue( sum_k A[m, k] * B[n, k] + bias[n] )
//
// Dense (sparse_linear, src/sparse.cpp:337-451): A is x [M, K] (bf16/f16), loaded
// by TMA.  Gather (sparse_submanifold_conv3d, src/sparse.cpp:999-1055): the K
// loop runs over 27 taps x Cin/64 blocks, A rows of tap t are x[nbr[t][m]]
// gathered with cp.async into the same 128B-swizzled layout TMA produces
// (missing neighbour = zero fill), B = W[t] [Cout, Cin] by TMA.
//
// CTA = 9 warps (13 for the gather variant), one CTA per SM, persistent over
// output tiles (n fastest so concurrently running CTAs share A tiles through L2):
//   warps 0-3  producers: thread 0 issues TMA; the gather variant adds
//              warps 9-12 and all 8 producer warps issue the row gathers
//              (cp.async, 16 rows per warp, 4 x 16 B per lane per stage)
//   warps 4-7  epilogue: tcgen05.ld 32 lanes x 32 columns per warp, bias /
//              activation / gate, staged in shared memory and written by TMA
//              box stores (the residual by TMA reduce-add)
//   warp  8    TMEM allocator + single-thread tcgen05.mma issuer
// Tile 128 x BN (BN in {64,128,256}), BK = 64 (one 128-byte swizzle atom),
// UMMA 128 x BN x 16; accumulators double-buffered in TMEM (2*BN columns) so
// the epilogue of tile i overlaps the main loop of tile i+1.
// When N is a multiple of 256 the CTA-pair kernel runs instead: a cluster of
// two CTAs on two SMs computes a 256 x (NSUB*256) tile with
// tcgen05.mma.cta_group::2, each SM staging its own A rows and half of B, so
// each SM streams half the B bytes per FLOP from L2 (the conv's bound).
// Every mbarrier wait is bounded (p3d_common.cuh): a stuck pipeline latches
// P3D_ERR_TIMEOUT and the kernel still frees its TMEM and exits.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "p3d_common.cuh"

namespace p3d {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 9 * 32;
// The dense 1-CTA kernel: 8 epilogue warps (0-7, two per TMEM lane quarter,
// each taking half of the tile's columns), the MMA warp 8, the producer warp 9.
constexpr int kThreadsD = 10 * 32;
// The gather variants add 4 producer warps (9-12): one producer warp per stage
// slot, up to 8 stages.
constexpr int kThreadsG = 13 * 32;
constexpr int kMmaWarp = 8;

struct GemmParams {
    const uint16_t *x;  // gather variant: base of x [n][cin] (16-bit elements)
    int64_t ldx;
    const int32_t *nbr;  // [27][M] or null
    const float *bias;
    void *out;
    int64_t ldo;
    const float *gate;
    int64_t gate_ld;
    const int32_t *batch_offsets;
    int nbatch;
    int64_t M, N, K;  // K = cin for gather
    int out_dtype;    // P3D_F32 / P3D_BF16 / P3D_F16
    uint32_t idesc;   // tcgen05 instruction descriptor (operand type, M, N)
    int epi;
    int *fault;
    // Per-head RMS norm + RoPE epilogue (head_dim 64): columns [0, norm_cols)
    // are normalised per 64-column head with gamma[col]; columns
    // [0, rope_cols) are then rotated with rope[pair][row] = (cos, sin)
    // (pair-major: a warp's 32 rows read one contiguous 256-byte run).
    int64_t norm_cols, rope_cols;
    const float *norm_gamma;
    const float2 *rope;
    // 1: the epilogue stages 32 x 32 boxes in shared memory and writes them
    // with TMA through tmap_o (store, or reduce-add for the residual).
    int tma_out;
    // Gather kernels: CTA (pair) c takes global steps [c T / G, (c+1) T / G)
    // of all tiles' T (tile, tap, K block) steps instead of whole tiles, so a
    // ragged last wave is spread over every CTA (pair).  A tile cut
    // between two CTAs is added into the f32 output by both (atomics; the
    // host zeroes the output first unless it accumulates a residual), the
    // bias by the part that holds its first step.
    int split;
    // Gather (pair kernel): per 256-row tile, bit t set when some row of the
    // tile has a neighbour at tap t; other taps are skipped (their A rows
    // are all zero).  Null: every tap.
    const uint32_t *tile_taps;
};

// TMA-store epilogue staging: each epilogue warp owns one or two 4 KB slots,
// each one 32-row x 128-byte box (32 f32 or 64 16-bit columns) in the
// 128-byte swizzle.  EPI_BYTES: the 4 warps x 2 slots of the pair kernel.
constexpr int EPI_SLOT_BYTES = 4096;
constexpr int EPI_WARP_BYTES = 2 * EPI_SLOT_BYTES;
constexpr int EPI_BYTES = 4 * EPI_WARP_BYTES;

// Shared memory for the operand stages of one CTA (the rest of the 227 KB
// holds the epilogue staging and the barriers).
constexpr int kStageBudget = 196608;

// 1-CTA tile: 128 x BN, BK = 64; accumulators double-buffered in TMEM.
// Dense tiles of 128 or 256 columns drain each accumulator with 8 epilogue
// warps of one staging slot each, keeping the operand stages of the 4-warp
// layout (measured on the trunk linears against two slots and one stage
// fewer: qkv + head norm + RoPE 50.7 vs 51.2 us, MLP down 58.6 vs 65.0 us);
// the gather and 64-column tiles with 4 warps of two slots.
template <int BN, bool GATHER>
struct Cfg {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EPI_WARPS = (!GATHER && BN >= 128) ? 8 : 4;
    static constexpr int EPI_SLOTS = EPI_WARPS == 8 ? 1 : 2;
    static constexpr int EPI_WARP_BYTES = EPI_SLOTS * EPI_SLOT_BYTES;
    static constexpr int EPI_BYTES = EPI_WARPS * EPI_WARP_BYTES;
    static constexpr int EPI_COLS = BN * 4 / EPI_WARPS;  // accumulator columns per epilogue warp
    static constexpr int BUDGET = EPI_WARPS == 8 ? 232448 - EPI_BYTES - 1024 - 256 : kStageBudget;
    static constexpr int STAGES = (BUDGET / STAGE_BYTES) > 8 ? 8 : (BUDGET / STAGE_BYTES);
    static constexpr int ACC_COLS = BN;
    static constexpr int ACC_BUFS = 2;
    static constexpr int TMEM_COLS = 2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512);
    static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + 1024 /*align*/ + 256 /*barriers*/;
    static_assert(SMEM <= 232448, "1-CTA GEMM shared memory");
};

// CTA-pair tile: 256 x (NSUB * 256).  Each CTA of the pair stages its own 128
// A rows and its 128-row half of each N = 256 slice of B, so the B stream per
// FLOP is half that of the 1-CTA tile; NSUB = 2 halves it again (one TMEM
// accumulator buffer of 512 columns, for long K loops such as the conv).
template <int NSUB>
struct Cfg2 {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_SUB = 128 * BK * 2;
    static constexpr int B_BYTES = NSUB * B_SUB;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (kStageBudget / STAGE_BYTES) > 8 ? 8 : (kStageBudget / STAGE_BYTES);
    static constexpr int ACC_COLS = NSUB * 256;
    static constexpr int ACC_BUFS = NSUB == 1 ? 2 : 1;
    static constexpr int TMEM_COLS = 512;
    static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + 1024 /*align*/ + 512 /*barriers*/;
};

template <typename T>
__device__ __forceinline__ void store16(T *o, const float (&v)[32], int ncols) {
    if (ncols == 32 && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
            uint4 pk;
            pk.x = pack2<T>(v[i], v[i + 1]);
            pk.y = pack2<T>(v[i + 2], v[i + 3]);
            pk.z = pack2<T>(v[i + 4], v[i + 5]);
            pk.w = pack2<T>(v[i + 6], v[i + 7]);
            *reinterpret_cast<uint4 *>(o + i) = pk;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i < ncols) o[i] = from_f32<T>(v[i]);
    }
}

__device__ __forceinline__ void store_chunk(const GemmParams &p, int64_t row, int64_t col0, const float (&v)[32],
                                            int ncols) {
    // ncols <= 32 valid columns starting at col0.
    if (p.epi & P3D_EPI_RESIDUAL) {
        float *o = reinterpret_cast<float *>(p.out) + row * p.ldo + col0;
        const float *g = nullptr;
        if (p.gate) {
            const int b = batch_of_row(p.batch_offsets, p.nbatch, row);
            g = p.gate + static_cast<int64_t>(b) * p.gate_ld + col0;
        }
        if (ncols == 32 && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
            // All 8 residual (and gate) loads are issued before any store so
            // they overlap: one DRAM round trip per chunk, not eight.
            float4 cur[8], gg[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) cur[i] = __ldcg(reinterpret_cast<const float4 *>(o) + i);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                gg[i] = g ? __ldg(reinterpret_cast<const float4 *>(g) + i) : make_float4(1.f, 1.f, 1.f, 1.f);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                cur[i].x += gg[i].x * v[4 * i];
                cur[i].y += gg[i].y * v[4 * i + 1];
                cur[i].z += gg[i].z * v[4 * i + 2];
                cur[i].w += gg[i].w * v[4 * i + 3];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) reinterpret_cast<float4 *>(o)[i] = cur[i];
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (i < ncols) o[i] += (g ? g[i] : 1.0f) * v[i];
        }
        return;
    }
    if (p.out_dtype == P3D_BF16) {
        store16<__nv_bfloat16>(reinterpret_cast<__nv_bfloat16 *>(p.out) + row * p.ldo + col0, v, ncols);
    } else if (p.out_dtype == P3D_F16) {
        store16<__half>(reinterpret_cast<__half *>(p.out) + row * p.ldo + col0, v, ncols);
    } else {
        float *o = reinterpret_cast<float *>(p.out) + row * p.ldo + col0;
        if (ncols == 32 && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4 *>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (i < ncols) o[i] = v[i];
        }
    }
}

// Epilogue of a partial tile (split schedule): lane l owns output row `row`;
// the f32 partial sums (+ bias when add_bias, times the row's gate for a
// residual epilogue) are added into the f32 output with vector atomics.
template <int COLS>
__device__ __forceinline__ void epilogue_rows_atomic(const GemmParams &p, uint32_t tacc, int64_t row, int64_t n0,
                                                     bool add_bias) {
#pragma unroll 1
    for (int cs = 0; cs < COLS; cs += 32) {
        float v[32];
        tmem_ld32(tacc + cs, v);
        tmem_ld_wait();
        const int64_t col0 = n0 + cs;
        if (col0 < p.N && row < p.M) {
            const int ncols = static_cast<int>(p.N - col0 < 32 ? p.N - col0 : 32);
            if (add_bias && p.bias) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] += (i < ncols) ? __ldg(p.bias + col0 + i) : 0.0f;
            }
            if ((p.epi & P3D_EPI_RESIDUAL) && p.gate) {
                const float *g = p.gate + static_cast<int64_t>(batch_of_row(p.batch_offsets, p.nbatch, row)) * p.gate_ld + col0;
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] *= (i < ncols) ? __ldg(g + i) : 0.0f;
            }
            float *o = reinterpret_cast<float *>(p.out) + row * p.ldo + col0;
            if (ncols == 32 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                    atomicAdd(reinterpret_cast<float4 *>(o + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (i < ncols) atomicAdd(o + i, v[i]);
            }
        }
        __syncwarp();  // reconverge before the next tcgen05.ld (.sync.aligned)
    }
}

// Epilogue of one warp for one accumulator buffer: lane l owns output row
// `row`; tacc addresses this warp's TMEM lane quarter at accumulator column
// 0; accumulator column c is output column n0 + c.  Bias, then per-head RMS
// norm + RoPE (64-column heads) or the activation, then the store / gated
// residual add.  Every tcgen05.ld is issued by the whole (converged) warp.
template <int COLS, bool HEADNORM>
__device__ __forceinline__ void epilogue_rows(const GemmParams &p, uint32_t tacc, int64_t row, int64_t n0) {
    if (HEADNORM && (p.norm_cols > 0 || p.rope_cols > 0)) {
#pragma unroll 1
        for (int cs = 0; cs < COLS; cs += 64) {
            float v[64];
            {
                float a[32], b[32];
                tmem_ld32(tacc + cs, a);
                tmem_ld32(tacc + cs + 32, b);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    v[i] = a[i];
                    v[32 + i] = b[i];
                }
            }
            const int64_t col0 = n0 + cs;
            if (col0 < p.N && row < p.M) {
                if (p.bias) {
#pragma unroll
                    for (int i = 0; i < 64; ++i) v[i] += __ldg(p.bias + col0 + i);
                }
                if (col0 < p.norm_cols) {
                    float ss = 0.0f;
#pragma unroll
                    for (int i = 0; i < 64; ++i) ss += v[i] * v[i];
                    const float inv = 8.0f / fmaxf(sqrtf(ss), 1e-12f);  // sqrt(64) / max(||v||, eps)
#pragma unroll
                    for (int i = 0; i < 64; ++i) v[i] = v[i] * inv * __ldg(p.norm_gamma + col0 + i);
                }
                if (col0 < p.rope_cols) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float2 r = __ldg(p.rope + static_cast<int64_t>(i) * p.M + row);
                        const float e = v[2 * i], o = v[2 * i + 1];
                        v[2 * i] = e * r.x - o * r.y;
                        v[2 * i + 1] = e * r.y + o * r.x;
                    }
                }
                float lo[32], hi[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    lo[i] = v[i];
                    hi[i] = v[32 + i];
                }
                store_chunk(p, row, col0, lo, 32);
                store_chunk(p, row, col0 + 32, hi, 32);
            }
            __syncwarp();
        }
        return;
    }
#pragma unroll 1
    for (int cs = 0; cs < COLS; cs += 32) {
        float v[32];
        tmem_ld32(tacc + cs, v);
        tmem_ld_wait();
        const int64_t col0 = n0 + cs;
        if (col0 < p.N && row < p.M) {
            const int ncols = static_cast<int>(p.N - col0 < 32 ? p.N - col0 : 32);
            if (p.bias) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] += (i < ncols) ? __ldg(p.bias + col0 + i) : 0.0f;
            }
            if (p.epi & P3D_EPI_GELU_TANH) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = gelu_tanh_f(v[i]);
            } else if (p.epi & P3D_EPI_SILU) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = silu_f(v[i]);
            }
            store_chunk(p, row, col0, v, ncols);
        }
        __syncwarp();  // reconverge before the next tcgen05.ld (.sync.aligned)
    }
}

// v[i] += b[i] for a warp-uniform 32-column vector (bias, gamma): float4
// loads when the vector is 16-byte aligned and whole.
__device__ __forceinline__ void add_vec32(float (&v)[32], const float *b, int ncols) {
    if (ncols == 32 && (reinterpret_cast<uintptr_t>(b) & 15) == 0) {
#pragma unroll
        for (int h = 0; h < 8; h += 4) {  // 4 vector loads in flight at a time
            float4 t[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) t[i] = __ldg(reinterpret_cast<const float4 *>(b) + h + i);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[4 * (h + i)] += t[i].x;
                v[4 * (h + i) + 1] += t[i].y;
                v[4 * (h + i) + 2] += t[i].z;
                v[4 * (h + i) + 3] += t[i].w;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i < ncols) v[i] += __ldg(b + i);
    }
}

__device__ __forceinline__ void mul_vec32(float (&v)[32], const float *g, int ncols) {
    if (ncols == 32 && (reinterpret_cast<uintptr_t>(g) & 15) == 0) {
#pragma unroll
        for (int h = 0; h < 8; h += 4) {  // 4 vector loads in flight at a time
            float4 t[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) t[i] = __ldg(reinterpret_cast<const float4 *>(g) + h + i);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[4 * (h + i)] *= t[i].x;
                v[4 * (h + i) + 1] *= t[i].y;
                v[4 * (h + i) + 2] *= t[i].z;
                v[4 * (h + i) + 3] *= t[i].w;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i < ncols) v[i] *= __ldg(g + i);
    }
}

// Staging slot for the next box: wait until the box last issued from this
// slot (two boxes ago) has been read by the TMA unit.
template <int SLOTS>
__device__ __forceinline__ uint8_t *acquire_slot(uint8_t *wbuf, int slot, int lane) {
    if (lane == 0) bulk_wait_read<SLOTS - 1>();
    __syncwarp();
    return wbuf + slot * EPI_SLOT_BYTES;
}

// This lane's 32 values as row `lane` of the slot, in the 128-byte swizzle
// (16-byte chunk c of a 128-byte row at c ^ (row & 7)).  f32: the whole
// 128-byte row; 16-bit: half `half` (columns 32*half .. +31) of a 64-column row.
__device__ __forceinline__ void stage_row(int out_dtype, uint8_t *buf, int lane, const float (&v)[32], int half) {
    uint8_t *rowp = buf + lane * 128;
    if (out_dtype == P3D_F32) {
#pragma unroll
        for (int c = 0; c < 8; ++c)
            *reinterpret_cast<float4 *>(rowp + ((c ^ (lane & 7)) << 4)) =
                make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
        return;
    }
    const bool bf = out_dtype == P3D_BF16;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint4 pk;
        pk.x = bf ? pack2<__nv_bfloat16>(v[8 * c], v[8 * c + 1]) : pack2<__half>(v[8 * c], v[8 * c + 1]);
        pk.y = bf ? pack2<__nv_bfloat16>(v[8 * c + 2], v[8 * c + 3]) : pack2<__half>(v[8 * c + 2], v[8 * c + 3]);
        pk.z = bf ? pack2<__nv_bfloat16>(v[8 * c + 4], v[8 * c + 5]) : pack2<__half>(v[8 * c + 4], v[8 * c + 5]);
        pk.w = bf ? pack2<__nv_bfloat16>(v[8 * c + 6], v[8 * c + 7]) : pack2<__half>(v[8 * c + 6], v[8 * c + 7]);
        *reinterpret_cast<uint4 *>(rowp + (((4 * half + c) ^ (lane & 7)) << 4)) = pk;
    }
}

// Lane 0 writes the staged 32-row box at (col0, row0): a TMA store, or (the
// residual epilogue, or part of a tile cut by the split schedule) a TMA
// reduce-add into the f32 output.  Rows >= M and columns >= N of the box are
// clipped by the tensor map's bounds.
template <int SLOTS>
__device__ __forceinline__ void issue_box(const CUtensorMap *tmo, const uint8_t *buf, int lane, int64_t col0,
                                          int64_t row0, int &slot, bool reduce) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        if (reduce)
            tma_reduce_add_2d(tmo, buf, static_cast<int>(col0), static_cast<int>(row0));
        else
            tma_store_2d(tmo, buf, static_cast<int>(col0), static_cast<int>(row0));
        bulk_commit();
    }
    slot = SLOTS == 1 ? 0 : slot ^ 1;
}

// Bias (null: none), activation and residual gate of one 32-column chunk of
// row `row`; false when the chunk lies entirely at or beyond column N
// (warp-uniform).
__device__ __forceinline__ bool prep_chunk(const GemmParams &p, const float *bias, int64_t row, int64_t col0,
                                           float (&v)[32]) {
    if (col0 >= p.N) return false;
    const int ncols = static_cast<int>(p.N - col0 < 32 ? p.N - col0 : 32);
    if (bias) add_vec32(v, bias + col0, ncols);
    if (p.epi & P3D_EPI_GELU_TANH) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = gelu_tanh_f(v[i]);
    } else if (p.epi & P3D_EPI_SILU) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = silu_f(v[i]);
    }
    if ((p.epi & P3D_EPI_RESIDUAL) && p.gate) {
        const int b = batch_of_row(p.batch_offsets, p.nbatch, row);
        mul_vec32(v, p.gate + static_cast<int64_t>(b) * p.gate_ld + col0, ncols);
    }
    return true;
}

// Rotate the 16 (even, odd) pairs of v: pair i by (cos, sin) = (r[i].x, r[i].y).
__device__ __forceinline__ void rope_rotate16(float (&v)[32], const float2 (&r)[16]) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float e = v[2 * i], o = v[2 * i + 1];
        v[2 * i] = e * r[i].x - o * r[i].y;
        v[2 * i + 1] = e * r[i].y + o * r[i].x;
    }
}

// TMA-store epilogue of one warp for one accumulator buffer (rows row0 ..
// row0+31, accumulator columns [0, COLS) = output columns n0 + c).  Boxes
// are 32 rows x 128 bytes: 32 f32 columns, or 64 16-bit columns staged from
// two 32-column chunks.  The next chunk's tcgen05.ld is in flight while the
// current one is finished.  bias: p.bias, or null for a part of a cut tile
// that does not hold its first step; reduce: TMA reduce-add instead of store.
template <int COLS, bool HEADNORM, int SLOTS = 2>
__device__ __forceinline__ void epilogue_rows_tma(const GemmParams &p, const CUtensorMap *tmo, uint32_t tacc,
                                                  int64_t row0, int lane, int64_t n0, uint8_t *wbuf, int &slot,
                                                  const float *bias, bool reduce) {
    static_assert(COLS % 64 == 0, "epilogue column count");
    const int64_t row = row0 + lane;
    const bool f32 = p.out_dtype == P3D_F32;
    float a[32], b[32];
    if (HEADNORM && (p.norm_cols > 0 || p.rope_cols > 0)) {
        // Per-head RMS norm + RoPE over 64-column heads (N % 64 == 0).  The
        // head's second half is read from TMEM twice (for the norm, then
        // for its output) so only one half plus its RoPE pairs stay live.
#pragma unroll 1
        for (int cs = 0; cs < COLS; cs += 64) {
            const int64_t col0 = n0 + cs;
            if (col0 >= p.N) break;  // warp-uniform
            __syncwarp();
            tmem_ld32(tacc + cs, a);
            tmem_ld32(tacc + cs + 32, b);
            const bool rope = col0 < p.rope_cols;
            const bool norm = col0 < p.norm_cols;
            const float2 *rp = p.rope + (row < p.M ? row : 0);  // pair j at rp[j * M]
            tmem_ld_wait_regs(a);
            tmem_ld_wait_regs(b);
            if (p.bias) {
                add_vec32(a, p.bias + col0, 32);
                add_vec32(b, p.bias + col0 + 32, 32);
            }
            float inv = 1.0f;
            if (norm) {
                float ss = 0.0f;
#pragma unroll
                for (int i = 0; i < 32; ++i) ss += a[i] * a[i] + b[i] * b[i];
                inv = 8.0f / fmaxf(sqrtf(ss), 1e-12f);  // sqrt(64) / max(||v||, eps)
            }
            uint8_t *buf = acquire_slot<SLOTS>(wbuf, slot, lane);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                if (half == 1) {
                    __syncwarp();
                    tmem_ld32(tacc + cs + 32, a);
                    tmem_ld_wait_regs(a);
                    if (p.bias) add_vec32(a, p.bias + col0 + 32, 32);
                    if (f32) buf = acquire_slot<SLOTS>(wbuf, slot, lane);
                }
                if (norm) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) a[i] *= inv;
                    mul_vec32(a, p.norm_gamma + col0 + 32 * half, 32);
                }
                if (rope) {
                    float2 r2[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) r2[i] = __ldg(rp + static_cast<int64_t>(16 * half + i) * p.M);
                    rope_rotate16(a, r2);
                }
                stage_row(p.out_dtype, buf, lane, a, f32 ? 0 : half);
                if (f32) issue_box<SLOTS>(tmo, buf, lane, col0 + 32 * half, row0, slot, reduce);
            }
            if (!f32) issue_box<SLOTS>(tmo, buf, lane, col0, row0, slot, reduce);
        }
        return;
    }
    __syncwarp();
    tmem_ld32(tacc, a);
    tmem_ld_wait_regs(a);
#pragma unroll 1
    for (int cs = 0; cs < COLS; cs += 64) {
        const int64_t col0 = n0 + cs;
        const bool more = cs + 64 < COLS;
        __syncwarp();
        tmem_ld32(tacc + cs + 32, b);
        uint8_t *buf = acquire_slot<SLOTS>(wbuf, slot, lane);
        const bool any = prep_chunk(p, bias, row, col0, a);
        if (any) {
            stage_row(p.out_dtype, buf, lane, a, 0);
            if (f32) issue_box<SLOTS>(tmo, buf, lane, col0, row0, slot, reduce);
        }
        tmem_ld_wait_regs(b);
        if (more) {
            __syncwarp();
            tmem_ld32(tacc + cs + 64, a);
        }
        if (f32) buf = acquire_slot<SLOTS>(wbuf, slot, lane);
        if (prep_chunk(p, bias, row, col0 + 32, b)) {
            stage_row(p.out_dtype, buf, lane, b, f32 ? 0 : 1);
            if (f32) issue_box<SLOTS>(tmo, buf, lane, col0 + 32, row0, slot, reduce);
        }
        if (!f32 && any) issue_box<SLOTS>(tmo, buf, lane, col0, row0, slot, reduce);
        if (more) tmem_ld_wait_regs(a);
    }
}

// Residual epilogues read-modify-write the f32 output: pull this lane's row
// segment into L2 while the tile's MMAs run, so the epilogue's loads hit L2.
__device__ __forceinline__ void prefetch_residual(const GemmParams &p, int64_t row, int64_t n0, int cols) {
    if (!(p.epi & P3D_EPI_RESIDUAL) || row >= p.M || n0 >= p.N) return;
    const float *rp = reinterpret_cast<const float *>(p.out) + row * p.ldo + n0;
    const int64_t c = p.N - n0 < cols ? p.N - n0 : cols;
    const uint32_t bytes = static_cast<uint32_t>(c * 4) & ~15u;
    if (bytes == 0 || (reinterpret_cast<uintptr_t>(rp) & 15) != 0) return;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(rp), "r"(bytes) : "memory");
}

// Warp-uniform bounded wait: lane 0 polls, the warp follows its verdict.
template <bool CLUSTER>
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, int *fault) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0)
        ok = (CLUSTER ? mbar_wait_cluster(bar, parity, fault) : mbar_wait(bar, parity, fault)) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <int BN, bool GATHER>
__global__ void __launch_bounds__(GATHER ? kThreadsG : kThreadsD, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_o, const GemmParams p) {
    using C = Cfg<BN, GATHER>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t *smem_a = smem;
    uint8_t *smem_b = smem + STAGES * C::A_BYTES;
    uint8_t *smem_o = smem_b + STAGES * C::B_BYTES;  // epilogue staging, C::EPI_BYTES
    uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem_o + C::EPI_BYTES);
    uint64_t *empty_bar = full_bar + STAGES;
    uint64_t *tfull_bar = empty_bar + STAGES;  // [2]
    uint64_t *tempty_bar = tfull_bar + 2;      // [2]
    uint64_t *done_bar = tempty_bar + 2;       // [1]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done_bar + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    const int64_t m_tiles = (p.M + BM - 1) / BM;
    const int64_t n_tiles = (p.N + BN - 1) / BN;
    const int64_t num_tiles = m_tiles * n_tiles;
    const int kblocks_per_tap = static_cast<int>((p.K + BK - 1) / BK);
    const int num_kb = GATHER ? 27 * kblocks_per_tap : kblocks_per_tap;
    // This CTA's work as units (tile, K steps [kb0, kb1)) in order: whole
    // tiles blockIdx.x + i * gridDim.x.  Split: the full waves (tiles below
    // r0 = floor(tiles / G) * G) stay whole tiles in that order, and the last,
    // ragged wave's steps are cut into G equal contiguous ranges, range b for
    // CTA b ([s_lo, s_hi), counted from tile r0's first step).
    const bool split = GATHER && p.split;
    const int64_t r0 = split ? (num_tiles / gridDim.x) * gridDim.x : num_tiles;
    const int64_t tail_steps = (num_tiles - r0) * num_kb;
    const int64_t s_lo = tail_steps * blockIdx.x / gridDim.x;
    const int64_t s_hi = tail_steps * (blockIdx.x + 1) / gridDim.x;
    struct Unit {
        int64_t tile;
        int kb0, kb1;
    };
    auto tail_unit = [&](Unit &u) -> bool {
        if (s_lo >= s_hi) return false;
        u.tile = r0 + s_lo / num_kb;
        u.kb0 = static_cast<int>(s_lo % num_kb);
        u.kb1 = static_cast<int>(std::min<int64_t>(num_kb, u.kb0 + (s_hi - s_lo)));
        return true;
    };
    auto first_unit = [&](Unit &u) -> bool {
        u.tile = blockIdx.x;
        u.kb0 = 0;
        u.kb1 = num_kb;
        if (u.tile < r0) return true;
        return split ? tail_unit(u) : false;
    };
    auto next_unit = [&](Unit &u) -> bool {
        if (u.tile >= r0) {  // last wave (split only)
            const int64_t g = (u.tile - r0 + 1) * num_kb;  // the next unit starts a tile
            if (u.kb1 < num_kb || g >= s_hi) return false;
            u.tile += 1;
            u.kb0 = 0;
            u.kb1 = static_cast<int>(std::min<int64_t>(num_kb, s_hi - g));
            return true;
        }
        u.tile += gridDim.x;
        if (u.tile < r0) return true;
        return split ? tail_unit(u) : false;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], C::EPI_WARPS);
        }
        mbar_init(done_bar, 1);
        fence_barrier_init();
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();     // the previous kernel's outputs (our inputs) are complete from here
    pdl_trigger();  // every CTA of this persistent grid is resident: the next kernel may queue

    // roles: gather: producers warps 0-3 and 9-12, epilogue 4-7; dense:
    // producer warp 9, epilogue 0-7 (4-7 for 64-column tiles); MMA warp 8
    const bool producer = GATHER ? (warp < 4 || warp > kMmaWarp) : warp == kMmaWarp + 1;
    const bool epilogue = warp < 8 && (C::EPI_WARPS == 8 || warp >= 4);
    if (producer) {
        // ------------------------------------------------------------ producer
        // gather: producer pw (warps 0-3 -> 0-3, 9-12 -> 4-7) issues the steps
        // s with s % 8 == pw; dense: lane 0 of warp 9 issues every TMA load
        const int t = GATHER ? (warp < 4 ? threadIdx.x : 0) : lane;
        const int pw = warp < 4 ? warp : warp - (kMmaWarp + 1) + 4;
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        bool return_early = false;  // gather: a producer warp without a stage slot
        if constexpr (GATHER) {
            // One producer warp per stage slot: this CTA's step s (a tap and
            // K block of one of its units, in unit order) goes to producer
            // warp s % STAGES (warps past STAGES stay idle), so the fixed cost
            // of a step (the empty wait, the barrier arrive, the index
            // bookkeeping) of STAGES steps overlaps; with cin = 64 a step is
            // one 128 x 64 x 64 MMA, far shorter than that cost.  Each warp
            // owns one slot and walks its rounds in order, so its parity
            // waits never alias an older phase.  Lane l gathers tile rows
            // [4 l, 4 l + 4) with one TMA tile::gather4 from x; a source
            // index outside [0, M) (the sentinel M, or -1 past the last row)
            // reads TMA's zero fill.  Row indices are loaded two of this
            // warp's steps (2 * STAGES steps) ahead into two fixed registers.
            static_assert(STAGES <= 8, "one producer warp per stage slot");
            if (pw >= STAGES) return_early = true;
            struct Pos {
                Unit u;
                int w;  // step within the tile: tap * kblocks_per_tap + K block
                int64_t m0, n0;
                bool valid;
            };
            auto place = [&](Pos &ps) {
                ps.m0 = (ps.u.tile / n_tiles) * BM;
                ps.n0 = (ps.u.tile % n_tiles) * BN;
            };
            auto advance = [&](Pos &ps, int by) {  // by < 27 <= the steps of a whole tile
                ps.w += by;
                while (ps.valid && ps.w >= ps.u.kb1) {
                    const int over = ps.w - ps.u.kb1;
                    ps.valid = next_unit(ps.u);
                    if (ps.valid) {
                        ps.w = ps.u.kb0 + over;
                        place(ps);
                    }
                }
            };
            auto load4 = [&](const Pos &ps) -> int4 {
                int r[4] = {-1, -1, -1, -1};
                if (ps.valid) {
                    const int64_t tap = ps.w / kblocks_per_tap;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int64_t row = ps.m0 + 4 * lane + j;
                        if (row < p.M) r[j] = __ldg(p.nbr + tap * p.M + row);
                    }
                }
                return make_int4(r[0], r[1], r[2], r[3]);
            };
            Pos pc;
            pc.valid = first_unit(pc.u);
            pc.w = pc.u.kb0;
            place(pc);
            advance(pc, pw);
            Pos pa = pc;
            const int4 first0 = load4(pa);
            advance(pa, STAGES);
            const int4 first1 = load4(pa);
            advance(pa, STAGES);
            int4 ring0 = first0, ring1 = first1;
            int64_t st = pw;  // this CTA's step index: stage st % STAGES, round st / STAGES
            while (pc.valid && ok && !return_early) {
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    if (!pc.valid || !ok) break;
                    int4 src;
                    if (u == 0) {
                        src = ring0;
                        ring0 = load4(pa);
                    } else {
                        src = ring1;
                        ring1 = load4(pa);
                    }
                    advance(pa, STAGES);
                    const int stg = static_cast<int>(st % STAGES);
                    const uint32_t ph = static_cast<uint32_t>((st / STAGES) & 1);
                    if (!warp_wait<false>(&empty_bar[stg], ph ^ 1, p.fault)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem_a + stg * C::A_BYTES;
                    uint8_t *sb = smem_b + stg * C::B_BYTES;
                    const int tap = pc.w / kblocks_per_tap;
                    const int kc = (pc.w - tap * kblocks_per_tap) * BK;
                    if (lane == 0) mbar_arrive_expect_tx(&full_bar[stg], C::A_BYTES + C::B_BYTES);
                    __syncwarp();
                    tma_gather4(sa + lane * 4 * 128, &tmap_a, &full_bar[stg], kc, src.x, src.y, src.z, src.w);
                    // Tap t's weights are rows [t*N, (t+1)*N) of the stacked [27*N, K] map.
                    if (lane == 0)
                        tma_load_2d(sb, &tmap_b, &full_bar[stg], kc, static_cast<int>(tap * p.N + pc.n0));
                    advance(pc, STAGES);
                    st += STAGES;
                }
            }
        } else {
            Unit un;
            for (bool more = first_unit(un); more && ok; more = next_unit(un)) {
                const int64_t m0 = (un.tile / n_tiles) * BM;
                const int64_t n0 = (un.tile % n_tiles) * BN;
                for (int kb = un.kb0; kb < un.kb1; ++kb) {
                    if (t == 0) {
                        if (!mbar_wait(&empty_bar[stage], phase ^ 1, p.fault)) {
                            ok = false;
                            break;
                        }
                        uint8_t *sa = smem_a + stage * C::A_BYTES;
                        uint8_t *sb = smem_b + stage * C::B_BYTES;
                        mbar_arrive_expect_tx(&full_bar[stage], C::A_BYTES + C::B_BYTES);
                        tma_load_2d(sa, &tmap_a, &full_bar[stage], kb * BK, static_cast<int>(m0));
                        tma_load_2d(sb, &tmap_b, &full_bar[stage], kb * BK, static_cast<int>(n0));
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == kMmaWarp) {
        // ---------------------------------------------------------- MMA issue
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            bool issued = false;
            const uint32_t idesc = p.idesc;
            Unit un;
            for (bool more = first_unit(un); more && ok; more = next_unit(un)) {
                if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, p.fault)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * C::ACC_COLS;
                for (int kb = un.kb0; kb < un.kb1; ++kb) {
                    if (!mbar_wait(&full_bar[stage], phase, p.fault)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem_a + stage * C::A_BYTES);
                    const uint32_t b_addr = smem_u32(smem_b + stage * C::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        umma_f16(d_tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc,
                                 (kb > un.kb0 || kk > 0) ? 1u : 0u);
                    issued = true;
                    umma_commit(&empty_bar[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit(&tfull_bar[acc]);
                if (++acc == C::ACC_BUFS) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
            // Drain: make sure every issued MMA finished before TMEM is freed.
            if (issued) {
                umma_commit(done_bar);
                mbar_wait(done_bar, 0, p.fault);
            }
        }
        __syncwarp();
    } else if (epilogue) {
        // ----------------------------------------------------------- epilogue
        // warp w drains TMEM lane quarter w % 4, columns [h E, (h+1) E) of
        // the accumulator (E = C::EPI_COLS; h = w / 4 - 1 with 4 warps, w / 4 with 8)
        const int q = warp & 3;  // TMEM lane quarter accessible to this warp
        const int h = C::EPI_WARPS == 8 ? (warp >> 2) : 0;
        const int ew = C::EPI_WARPS == 8 ? warp : q;  // staging slot group
        constexpr int EC = C::EPI_COLS;
        int acc = 0;
        uint32_t acc_phase = 0;
        int slot = 0;
        Unit un;
        for (bool more = first_unit(un); more; more = next_unit(un)) {
            const int64_t tile = un.tile;
            const int64_t m0 = (tile / n_tiles) * BM;
            const int64_t n0 = (tile % n_tiles) * BN + h * EC;
            const bool whole = un.kb0 == 0 && un.kb1 == num_kb;
            if (!p.tma_out && whole) prefetch_residual(p, m0 + q * 32 + lane, n0, EC);
            if (!warp_wait<false>(&tfull_bar[acc], acc_phase, p.fault)) break;
            tc_fence_after();
            const uint32_t tacc =
                tmem_base + acc * C::ACC_COLS + h * EC + (static_cast<uint32_t>(q * 32) << 16);
            if (p.tma_out)  // a cut tile's part is reduce-added, the bias by the part holding step 0
                epilogue_rows_tma<EC, !GATHER, C::EPI_SLOTS>(
                    p, &tmap_o, tacc, m0 + q * 32, lane, n0, smem_o + ew * C::EPI_WARP_BYTES, slot,
                    (!GATHER || un.kb0 == 0) ? p.bias : nullptr, (GATHER && !whole) || (p.epi & P3D_EPI_RESIDUAL));
            else if (!whole)
                epilogue_rows_atomic<EC>(p, tacc, m0 + q * 32 + lane, n0, un.kb0 == 0);
            else
                epilogue_rows<EC, !GATHER>(p, tacc, m0 + q * 32 + lane, n0);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty_bar[acc]);
            if (++acc == C::ACC_BUFS) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (p.tma_out && lane == 0) bulk_wait_all();  // staging slots stay live until the stores land
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// CTA-pair (cluster of 2) variant: tcgen05.mma.cta_group::2 with M = 256, the
// even CTA (rank 0) issuing for both.  Per stage each CTA fills its own
// shared memory (A rows m0 + 128*rank, B rows of its half).  Both CTAs' TMA
// loads count their bytes on the even CTA's `full` barrier (the even CTA
// posts the expected bytes of both).  Gather variant: row gathers arrive on
// their own CTA's `full` barrier through cp.async.mbarrier.arrive, and the
// odd CTA's warp 8 forwards that completion to the even CTA's `full`
// barrier (release, cluster scope).  The issuer's tcgen05.commit arrives on the
// `empty` / `tfull` barriers of both CTAs (one commit per CTA,
// shared::cluster addresses); both epilogues release the accumulator to the
// even CTA's `tempty` barrier (count 8).  No TMA multicast.  All waits are
// bounded; the pair meets at cluster barriers before the first remote
// arrival and before freeing TMEM.
template <int NSUB, bool GATHER>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GATHER ? kThreadsG : kThreads, 1)
    gemm2_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const __grid_constant__ CUtensorMap tmap_o, const GemmParams p) {
    using C = Cfg2<NSUB>;
    constexpr int STAGES = C::STAGES;
    constexpr int PAIR_N = NSUB * 256;
    // Epilogue warps per CTA: with 4 stages (NSUB = 2) the 4 gather warps
    // 9-12 have no stage slot and drain the accumulator's second half, so
    // the MMA (one accumulator buffer) waits on half as long an epilogue;
    // one 4 KB staging slot each.  Otherwise warps 4-7 with two slots.
    constexpr int EPI_WARPS = (GATHER && STAGES + 4 <= 8 && NSUB == 2) ? 8 : 4;
    constexpr int EPI_SLOTS = EPI_WARPS == 8 ? 1 : 2;
    constexpr int EPI_COLS = C::ACC_COLS * 4 / EPI_WARPS;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t *smem_a = smem;
    uint8_t *smem_b = smem + STAGES * C::A_BYTES;
    uint8_t *smem_o = smem_b + STAGES * C::B_BYTES;  // epilogue staging, EPI_BYTES
    uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem_o + EPI_BYTES);
    uint64_t *empty_bar = full_bar + STAGES;
    uint64_t *tfull_bar = empty_bar + STAGES;  // [2]
    uint64_t *tempty_bar = tfull_bar + 2;      // [2]
    uint64_t *done_bar = tempty_bar + 2;       // [1]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done_bar + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const int64_t pair = blockIdx.x >> 1;
    const int64_t npairs = gridDim.x >> 1;

    const int64_t m_tiles = (p.M + 2 * BM - 1) / (2 * BM);
    const int64_t n_tiles = (p.N + PAIR_N - 1) / PAIR_N;
    const int64_t num_tiles = m_tiles * n_tiles;
    const int kblocks_per_tap = static_cast<int>((p.K + BK - 1) / BK);
    const int num_kb = GATHER ? 27 * kblocks_per_tap : kblocks_per_tap;
    // taps of a pair tile (the centre tap always: every row has itself)
    auto tile_taps = [&](int64_t tile) -> uint32_t {
        if (!GATHER || !p.tile_taps) return 0x7FFFFFFu;
        return (__ldg(p.tile_taps + tile / n_tiles) | (1u << 13)) & 0x7FFFFFFu;
    };
    auto tile_kb = [&](int64_t tile) -> int { return GATHER ? __popc(tile_taps(tile)) * kblocks_per_tap : num_kb; };
    // This pair's work as units (tile, steps [kb0, kb1) of the tile's used
    // taps x K blocks), in order: whole tiles pair + i * npairs.  Split: the
    // full waves (tiles below r0 = floor(tiles / pairs) * pairs) stay whole
    // tiles in that order, so all pairs stream the same taps' weights and
    // nearby rows at a time, and the last, ragged wave's tiles are cut into
    // equal contiguous step ranges, one per pair (split_info, found by warp 0
    // below).
    const bool split = GATHER && p.split;
    const int64_t r0 = split ? (num_tiles / npairs) * npairs : num_tiles;
    int64_t *split_info = reinterpret_cast<int64_t *>(done_bar + 2);  // {tile, kb, first step, end step}
    struct Unit {
        int64_t tile;
        int kb0, kb1;
        int64_t g0;  // last wave: index of step kb0 among the last wave's steps
    };
    auto tail_unit = [&](Unit &u) -> bool {
        u.tile = split_info[0];
        if (u.tile >= num_tiles) return false;
        u.kb0 = static_cast<int>(split_info[1]);
        u.g0 = split_info[2];
        u.kb1 = static_cast<int>(std::min<int64_t>(tile_kb(u.tile), u.kb0 + (split_info[3] - u.g0)));
        return true;
    };
    auto first_unit = [&](Unit &u) -> bool {
        u.tile = pair;
        u.kb0 = 0;
        u.g0 = 0;
        if (u.tile >= r0) return split ? tail_unit(u) : false;
        u.kb1 = tile_kb(u.tile);
        return true;
    };
    auto next_unit = [&](Unit &u) -> bool {
        if (u.tile >= r0) {  // last wave (split only)
            const int64_t g = u.g0 + (u.kb1 - u.kb0);
            if (u.kb1 < tile_kb(u.tile) || g >= split_info[3] || u.tile + 1 >= num_tiles) return false;
            u.tile += 1;
            u.kb0 = 0;
            u.g0 = g;
            u.kb1 = static_cast<int>(std::min<int64_t>(tile_kb(u.tile), split_info[3] - g));
            return true;
        }
        u.tile += npairs;
        if (u.tile >= r0) return split ? tail_unit(u) : false;
        u.kb1 = tile_kb(u.tile);
        return true;
    };
    if (split && warp == 0) {
        pdl_wait();
        // the last wave's steps T, then this pair's range [T p / P, T (p+1) / P)
        // and the tile and step where it starts (warp-wide scan over the masks)
        int64_t total = 0;
#pragma unroll 4
        for (int64_t t = r0 + lane; t < num_tiles; t += 32) total += tile_kb(t);  // independent loads
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
        const int64_t s_lo = total * pair / npairs, s_hi = total * (pair + 1) / npairs;
        int64_t base = 0, t_lo = num_tiles, k_lo = 0;
        for (int64_t c = r0; c < num_tiles && t_lo == num_tiles; c += 32) {
            const int64_t t = c + lane;
            const int v = t < num_tiles ? tile_kb(t) : 0;
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const unsigned hit = __ballot_sync(0xffffffffu, t < num_tiles && base + incl > s_lo);
            if (hit) {
                const int l = __ffs(hit) - 1;
                const int incl_l = __shfl_sync(0xffffffffu, incl, l), v_l = __shfl_sync(0xffffffffu, v, l);
                t_lo = c + l;
                k_lo = s_lo - (base + incl_l - v_l);
            }
            base += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) {
            split_info[0] = s_lo < s_hi ? t_lo : num_tiles;
            split_info[1] = k_lo;
            split_info[2] = s_lo;
            split_info[3] = s_hi;
        }
    }

    if (threadIdx.x == 0) {
        // full: the even CTA's expect_tx arrival; both CTAs' TMA bytes complete on it
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], 2 * EPI_WARPS);
        }
        mbar_init(done_bar, 1);
        fence_barrier_init();
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
    }
    if (warp == kMmaWarp) {
        tmem_alloc2(tmem_slot, C::TMEM_COLS);
        tmem_relinquish2();
    }
    tc_fence_before();
    cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();
    pdl_trigger();

    const bool epilogue2 = EPI_WARPS == 8 && warp > kMmaWarp;  // second epilogue group
    if ((warp < 4 || (GATHER && warp > kMmaWarp)) && !epilogue2) {
        // ------------------------------------------------------------ producer
        const int pw = warp < 4 ? warp : warp - (kMmaWarp + 1) + 4;
        bool ok = true;
        if constexpr (GATHER) {
            // One producer warp per stage slot (pw < STAGES), as in the 1-CTA
            // gather: step s = (pair tile, used tap, K block) goes to warp
            // s % STAGES, which fills this CTA's 128 A rows of the stage with
            // one tile::gather4 per lane (rows m0 + 4 lane .. + 3; a source
            // outside [0, M) reads zeros) and its half of B with 2D loads.
            // Both CTAs' bytes complete on the even CTA's `full` barrier, whose
            // expect_tx the even CTA posts for both.  Taps no row of the tile
            // uses are skipped (the step's tap is the (w / kpt)-th set bit of
            // the tile's mask).
            static_assert(STAGES <= 8, "one producer warp per stage slot");
            struct Pos {
                Unit u;
                int w;  // step within the tile's used taps x K blocks
                int64_t m0, n0;
                uint32_t mask;
                bool valid;
            };
            auto place = [&](Pos &ps) {
                ps.m0 = (ps.u.tile / n_tiles) * (2 * BM) + rank * BM;
                ps.n0 = (ps.u.tile % n_tiles) * PAIR_N;
                ps.mask = tile_taps(ps.u.tile);
            };
            auto advance = [&](Pos &ps, int by) {
                ps.w += by;
                while (ps.valid && ps.w >= ps.u.kb1) {
                    const int over = ps.w - ps.u.kb1;
                    ps.valid = next_unit(ps.u);
                    if (ps.valid) {
                        ps.w = ps.u.kb0 + over;
                        place(ps);
                    }
                }
            };
            auto tap_of = [&](const Pos &ps) -> int { return static_cast<int>(__fns(ps.mask, 0, ps.w / kblocks_per_tap + 1)); };
            auto load4 = [&](const Pos &ps) -> int4 {
                int r[4] = {-1, -1, -1, -1};
                if (ps.valid) {
                    const int64_t tap = tap_of(ps);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int64_t row = ps.m0 + 4 * lane + j;
                        if (row < p.M) r[j] = __ldg(p.nbr + tap * p.M + row);
                    }
                }
                return make_int4(r[0], r[1], r[2], r[3]);
            };
            if (pw < STAGES) {
                Pos pc;
                pc.valid = first_unit(pc.u);
                pc.w = pc.u.kb0;
                if (pc.valid) place(pc);
                advance(pc, pw);  // this warp's first step: the pair's step pw
                Pos pa = pc;
                const int4 first0 = load4(pa);
                advance(pa, STAGES);
                const int4 first1 = load4(pa);
                advance(pa, STAGES);
                int4 ring0 = first0, ring1 = first1;
                int64_t st = pw;  // the pair's step index: stage st % STAGES, round st / STAGES
                while (pc.valid && ok) {
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        if (!pc.valid || !ok) break;
                        int4 src;
                        if (u == 0) {
                            src = ring0;
                            ring0 = load4(pa);
                        } else {
                            src = ring1;
                            ring1 = load4(pa);
                        }
                        advance(pa, STAGES);
                        const int stg = static_cast<int>(st % STAGES);
                        const uint32_t ph = static_cast<uint32_t>((st / STAGES) & 1);
                        if (!warp_wait<true>(&empty_bar[stg], ph ^ 1, p.fault)) {
                            ok = false;
                            break;
                        }
                        uint8_t *sa = smem_a + stg * C::A_BYTES;
                        uint8_t *sb = smem_b + stg * C::B_BYTES;
                        const int tap = tap_of(pc);
                        const int kc = (pc.w % kblocks_per_tap) * BK;
                        const uint32_t fb = mapa_shared(smem_u32(&full_bar[stg]), 0);
                        if (rank == 0 && lane == 0) mbar_arrive_expect_tx(&full_bar[stg], 2 * (C::A_BYTES + C::B_BYTES));
                        __syncwarp();
                        tma_gather4_pair(sa + lane * 4 * 128, &tmap_a, fb, kc, src.x, src.y, src.z, src.w);
                        if (lane == 0) {
#pragma unroll
                            for (int j = 0; j < NSUB; ++j)
                                tma_load_2d_pair(sb + j * C::B_SUB, &tmap_b, fb, kc,
                                                 static_cast<int>(tap * p.N + pc.n0 + j * 256 + rank * 128));
                        }
                        advance(pc, STAGES);
                        st += STAGES;
                    }
                }
            }
        } else {
            const int t = threadIdx.x;
            int stage = 0;
            uint32_t phase = 0;
            for (int64_t tile = pair; tile < num_tiles && ok; tile += npairs) {
                const int64_t m0 = (tile / n_tiles) * (2 * BM) + rank * BM;
                const int64_t n0 = (tile % n_tiles) * PAIR_N;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (t == 0) {
                        if (!mbar_wait_cluster(&empty_bar[stage], phase ^ 1, p.fault)) {
                            ok = false;
                            break;
                        }
                        uint8_t *sa = smem_a + stage * C::A_BYTES;
                        uint8_t *sb = smem_b + stage * C::B_BYTES;
                        const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
                        if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * (C::A_BYTES + C::B_BYTES));
                        tma_load_2d_pair(sa, &tmap_a, fb, kb * BK, static_cast<int>(m0));
#pragma unroll
                        for (int j = 0; j < NSUB; ++j)
                            tma_load_2d_pair(sb + j * C::B_SUB, &tmap_b, fb, kb * BK,
                                             static_cast<int>(n0 + j * 256 + rank * 128));
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0 && rank == 0) {
            // ------------------------------------------------ pair MMA issue
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            bool issued = false;
            const uint32_t idesc = p.idesc;
            Unit un;
            for (bool more = first_unit(un); more && ok; more = next_unit(un)) {
                if (!mbar_wait_cluster(&tempty_bar[acc], acc_phase ^ 1, p.fault)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * C::ACC_COLS;
                for (int kb = un.kb0; kb < un.kb1; ++kb) {
                    if (!mbar_wait_cluster(&full_bar[stage], phase, p.fault)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem_a + stage * C::A_BYTES);
                    const uint32_t b_addr = smem_u32(smem_b + stage * C::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
#pragma unroll
                        for (int j = 0; j < NSUB; ++j)
                            umma2_f16(d_tmem + j * 256, sw128_desc(a_addr + kk * 32),
                                      sw128_desc(b_addr + j * C::B_SUB + kk * 32), idesc,
                                      (kb > un.kb0 || kk > 0) ? 1u : 0u);
                    issued = true;
                    const uint32_t e = smem_u32(&empty_bar[stage]);
                    umma_commit2(e);
                    umma_commit2(mapa_shared(e, peer));
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                const uint32_t f = smem_u32(&tfull_bar[acc]);
                umma_commit2(f);
                umma_commit2(mapa_shared(f, peer));
                if (++acc == C::ACC_BUFS) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
            if (issued) {
                umma_commit2(smem_u32(done_bar));
                mbar_wait(done_bar, 0, p.fault);
            }
        }
        __syncwarp();
    } else {
        // ----------------------------------------------------------- epilogue
        // warp w drains TMEM lane quarter w % 4, accumulator columns
        // [h E, (h+1) E) (E = EPI_COLS; h = 1 for the second group)
        const int q = warp & 3;
        const int h = epilogue2 ? 1 : 0;
        const int ew = h * 4 + q;  // staging slot group
        int acc = 0;
        uint32_t acc_phase = 0;
        int slot = 0;
        Unit un;
        for (bool more = first_unit(un); more; more = next_unit(un)) {
            const int64_t tile = un.tile;
            const int64_t m0 = (tile / n_tiles) * (2 * BM) + rank * BM;
            const int64_t n0 = (tile % n_tiles) * PAIR_N + h * EPI_COLS;
            const bool whole = un.kb0 == 0 && un.kb1 == tile_kb(tile);
            if (!p.tma_out && whole) prefetch_residual(p, m0 + q * 32 + lane, n0, EPI_COLS);
            if (!warp_wait<true>(&tfull_bar[acc], acc_phase, p.fault)) break;
            tc_fence_after();
            const uint32_t tacc =
                tmem_base + acc * C::ACC_COLS + h * EPI_COLS + (static_cast<uint32_t>(q * 32) << 16);
            if (p.tma_out)  // a cut tile's part is reduce-added, the bias by the part holding step 0
                epilogue_rows_tma<EPI_COLS, !GATHER, EPI_SLOTS>(p, &tmap_o, tacc, m0 + q * 32, lane, n0,
                                                                smem_o + ew * EPI_SLOTS * EPI_SLOT_BYTES, slot,
                                                                un.kb0 == 0 ? p.bias : nullptr,
                                                                !whole || (p.epi & P3D_EPI_RESIDUAL));
            else if (!whole)
                epilogue_rows_atomic<EPI_COLS>(p, tacc, m0 + q * 32 + lane, n0, un.kb0 == 0);
            else
                epilogue_rows<EPI_COLS, !GATHER>(p, tacc, m0 + q * 32 + lane, n0);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                const uint32_t te = smem_u32(&tempty_bar[acc]);
                if (rank == 0)
                    mbar_arrive(&tempty_bar[acc]);
                else
                    mbar_arrive_cluster(mapa_shared(te, peer));
            }
            if (++acc == C::ACC_BUFS) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (p.tma_out && lane == 0) bulk_wait_all();  // staging slots stay live until the stores land
    }

    __syncwarp();
    tc_fence_before();
    cluster_sync_all();  // no remote arrival or pair MMA is pending past here
    tc_fence_after();
    if (warp == kMmaWarp) tmem_dealloc2(tmem_base, C::TMEM_COLS);
}

using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode_fn() {
    static EncodeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeFn>(ptr);
    });
    return fn;
}

template <int BN, bool GATHER>
int launch_gemm(p3d_ctx *ctx, const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &to,
                const GemmParams &p) {
    using C = Cfg<BN, GATHER>;
    static bool attr_set = false;
    if (!attr_set) {
        P3D_CUDA(ctx, cudaFuncSetAttribute(gemm_tc_kernel<BN, GATHER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           C::SMEM));
        attr_set = true;
    }
    const int64_t tiles = ceil_div(p.M, BM) * ceil_div(p.N, BN);
    const int grid = static_cast<int>(std::min<int64_t>(tiles, ctx->num_sms));
    GemmParams q = p;
    q.split = 0;
    // Split schedule for a gather with a ragged last wave of 1-3 waves (e.g.
    // 171 tiles on 148 SMs): the last wave's tiles are cut into equal step
    // ranges, one per CTA, whose parts are summed into the f32 output (TMA
    // reduce-add, else atomics; the last wave's rows zeroed first unless a
    // residual is accumulated).  f32 outputs without an activation only.
    // (For the dense trunk linears the cut parts' extra epilogues cost more
    // than the ragged wave: out-projection 27 -> 36 us, MLP down 61 -> 66 us.)
    if (GATHER && tiles > grid && tiles < 4 * static_cast<int64_t>(grid) && tiles % grid != 0 &&
        p.out_dtype == P3D_F32 && !(p.epi & (P3D_EPI_GELU_TANH | P3D_EPI_SILU))) {
        q.split = 1;
        if (!(p.epi & P3D_EPI_RESIDUAL)) {
            const int64_t row0 = ((tiles / grid) * grid / ceil_div(p.N, BN)) * BM;
            P3D_CUDA(ctx, cudaMemset2DAsync(static_cast<float *>(p.out) + row0 * p.ldo, sizeof(float) * p.ldo, 0,
                                            sizeof(float) * p.N, p.M - row0, ctx->stream));
        }
    }
    P3D_CUDA(ctx, launch_pdl(gemm_tc_kernel<BN, GATHER>, dim3(grid), dim3(GATHER ? kThreadsG : kThreadsD), C::SMEM,
                             ctx->stream, ta, tb, to, q));
    return check_launch(ctx, "gemm_tc_kernel");
}

template <int NSUB, bool GATHER>
int launch_gemm2(p3d_ctx *ctx, const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &to,
                 const GemmParams &p) {
    using C = Cfg2<NSUB>;
    static bool attr_set = false;
    if (!attr_set) {
        P3D_CUDA(ctx, cudaFuncSetAttribute(gemm2_tc_kernel<NSUB, GATHER>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr_set = true;
    }
    // Persistent grid: as many pairs as can be co-resident (not every SM
    // can be paired into a cluster), so no pair waits for a second wave.
    static int max_pairs = 0;
    if (max_pairs == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (ctx->num_sms / 2), 1, 1);
        cfg.blockDim = dim3(GATHER ? kThreadsG : kThreads, 1, 1);
        cfg.dynamicSmemBytes = C::SMEM;
        cfg.stream = ctx->stream;
        int n = 0;
        P3D_CUDA(ctx, cudaOccupancyMaxActiveClusters(&n, gemm2_tc_kernel<NSUB, GATHER>, &cfg));
        max_pairs = std::max(1, std::min(n, ctx->num_sms / 2));
    }
    const int64_t tiles = ceil_div(p.M, 2 * BM) * ceil_div(p.N, NSUB * 256);
    const int pairs = static_cast<int>(std::min<int64_t>(tiles, max_pairs));
    GemmParams q = p;
    q.split = 0;
    // Split schedule for a ragged last wave (e.g. 342 pair tiles of the
    // config-2 fine level on 74 pairs: 46 pairs would run a fifth tile): each
    // pair runs 4 whole tiles, then an equal share of the last 46 tiles'
    // steps.  f32 output without an activation only, since cut tiles are
    // summed by atomics.
    if (GATHER && tiles > pairs && tiles % pairs != 0 && tiles < 16 * static_cast<int64_t>(pairs) &&
        p.out_dtype == P3D_F32 && !(p.epi & (P3D_EPI_GELU_TANH | P3D_EPI_SILU))) {
        q.split = 1;
        if (!(p.epi & P3D_EPI_RESIDUAL)) {
            // zero the rows of the last wave's tiles (the only ones cut)
            const int64_t n_tiles = ceil_div(p.N, NSUB * 256);
            const int64_t row0 = ((tiles / pairs) * pairs / n_tiles) * (2 * BM);
            P3D_CUDA(ctx, cudaMemset2DAsync(static_cast<float *>(p.out) + row0 * p.ldo, sizeof(float) * p.ldo, 0,
                                            sizeof(float) * p.N, p.M - row0, ctx->stream));
        }
    }
    P3D_CUDA(ctx, launch_pdl(gemm2_tc_kernel<NSUB, GATHER>, dim3(2 * pairs), dim3(GATHER ? kThreadsG : kThreads),
                             C::SMEM, ctx->stream, ta, tb, to, q));
    return check_launch(ctx, "gemm2_tc_kernel");
}

int pick_bn(int64_t n) {
    if (n <= 64) return 64;
    if (n <= 128) return 128;
    return 256;
}

// P3D_GEMM_TMA_STORE=0 selects the direct-store epilogue (lane = row,
// vector stores / read-modify-write residual) instead of the TMA one.
bool tma_store_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("P3D_GEMM_TMA_STORE");
        return !(e && e[0] == '0');
    }();
    return on;
}

// The TMA epilogue needs a 16-byte aligned output with a 16-byte row pitch
// and row coordinates that fit the map's int32 coordinates.
bool tma_out_ok(const GemmParams &p) {
    const int es = p.out_dtype == P3D_F32 ? 4 : 2;
    return (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 && (p.ldo * es) % 16 == 0 && p.M < (int64_t(1) << 31) &&
           p.N < (int64_t(1) << 31);
}

// Output map for the TMA epilogue: [M rows, N cols] at pitch ldo, boxes of
// 32 rows x 128 bytes (32 f32 or 64 16-bit columns) in the 128-byte swizzle,
// matching the staging layout of stage_row.
int make_tmap_out(p3d_ctx *ctx, CUtensorMap *map, void *base, int dtype, uint64_t rows, uint64_t cols, uint64_t ld) {
    EncodeFn fn = get_encode_fn();
    if (!fn) return set_error(ctx, P3D_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const bool f32 = dtype == P3D_F32;
    const uint64_t es = f32 ? 4 : 2;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * es};
    cuuint32_t box[2] = {f32 ? 32u : 64u, 32};  // 128-byte box rows
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                       : (dtype == P3D_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
    CUresult r = fn(map, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(ctx, P3D_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed: " + std::to_string(r));
    return P3D_OK;
}

// x == nullptr selects the gather (sparse conv) variant, whose B operand is
// the [27 * N, K] tap stack.  Builds the tensor maps and instruction
// descriptor for the chosen kernel and launches it.
int run_gemm(p3d_ctx *ctx, const void *x, int64_t ldx, const void *w, int ab_dtype, GemmParams p) {
    const bool gather = x == nullptr;
    const bool bf16 = ab_dtype == P3D_BF16;
    const int64_t w_rows = gather ? 27 * p.N : p.N;
    CUtensorMap ta, tb, to;
    std::memset(&to, 0, sizeof(to));
    p.tma_out = 0;
    if (tma_store_enabled() && tma_out_ok(p)) {
        int rc = make_tmap_out(ctx, &to, p.out, p.out_dtype, p.M, p.N, p.ldo);
        if (rc) return rc;
        p.tma_out = 1;
    }
    // The pair kernel serves the gather (conv) path, whose 27*Cin-long K loop
    // streams the most B bytes per output tile; for the dense linears
    // (K <= 4096) it measured no faster than the 1-CTA kernel on B200
    // (qkv 8184x3072x1024: 69.0 vs 69.0 us; MLP-up 99.5 vs 96.6 us).
    if (gather && p.N % 256 == 0) {
        // Two N = 256 MMAs per pair tile when N allows (the long K loop of a
        // conv hides the unbuffered epilogue).
        const int nsub = p.N % 512 == 0 ? 2 : 1;
        int rc = make_tmap_16bit_2d(ctx, &tb, w, ab_dtype, w_rows, p.K, p.K, 128);
        if (rc) return rc;
        // A rows by tile::gather4 from x [M][K] (box 64 columns x 1 row)
        if ((rc = make_tmap_16bit_2d(ctx, &ta, p.x, ab_dtype, p.M, p.K, p.ldx, 1))) return rc;
        p.idesc = idesc_f32acc(2 * BM, 256, bf16);
        return nsub == 2 ? launch_gemm2<2, true>(ctx, ta, tb, to, p) : launch_gemm2<1, true>(ctx, ta, tb, to, p);
    }
    const int bn = pick_bn(p.N);
    int rc = make_tmap_16bit_2d(ctx, &tb, w, ab_dtype, w_rows, p.K, p.K, bn);
    if (rc) return rc;
    // dense: A tiles of 128 rows; gather: A rows by tile::gather4 (box 64 x 1 row)
    if ((rc = gather ? make_tmap_16bit_2d(ctx, &ta, p.x, ab_dtype, p.M, p.K, p.ldx, 1)
                     : make_tmap_16bit_2d(ctx, &ta, x, ab_dtype, p.M, p.K, ldx, BM)))
        return rc;
    p.idesc = idesc_f32acc(BM, bn, bf16);
    if (gather) {
        if (bn == 64) return launch_gemm<64, true>(ctx, ta, tb, to, p);
        if (bn == 128) return launch_gemm<128, true>(ctx, ta, tb, to, p);
        return launch_gemm<256, true>(ctx, ta, tb, to, p);
    }
    if (bn == 64) return launch_gemm<64, false>(ctx, ta, tb, to, p);
    if (bn == 128) return launch_gemm<128, false>(ctx, ta, tb, to, p);
    return launch_gemm<256, false>(ctx, ta, tb, to, p);
}

}  // namespace

int make_tmap_16bit_2d(p3d_ctx *ctx, CUtensorMap *map, const void *base, int dtype, uint64_t rows, uint64_t cols,
                       uint64_t pitch_elems, uint32_t box_rows) {
    EncodeFn fn = get_encode_fn();
    if (!fn) return set_error(ctx, P3D_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (pitch_elems * 2) % 16 != 0)
        return set_error(ctx, P3D_ERR_INVALID, "TMA operand must be 16-byte aligned with a 16-byte row pitch");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch_elems * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt =
        dtype == P3D_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(ctx, P3D_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
    return P3D_OK;
}

}  // namespace p3d

using namespace p3d;

namespace {
int linear_impl(p3d_ctx *ctx, const void *x, int64_t ldx, const void *w, int ab_dtype, const float *bias, int64_t m,
                int64_t n, int64_t k, void *out, int64_t ldo, int out_dtype, int epilogue, const float *gate,
                int64_t gate_ld, const int32_t *batch_offsets, int nbatch, int64_t norm_cols, const float *norm_gamma,
                int64_t rope_cols, const float *rope);
}

extern "C" int p3d_linear(p3d_ctx *ctx, const void *x, int64_t ldx, const void *w, int ab_dtype, const float *bias,
                          int64_t m, int64_t n, int64_t k, void *out, int64_t ldo, int out_dtype, int epilogue,
                          const float *gate, int64_t gate_ld, const int32_t *batch_offsets, int nbatch) {
    return linear_impl(ctx, x, ldx, w, ab_dtype, bias, m, n, k, out, ldo, out_dtype, epilogue, gate, gate_ld,
                       batch_offsets, nbatch, 0, nullptr, 0, nullptr);
}

extern "C" int p3d_linear_headnorm(p3d_ctx *ctx, const void *x, int64_t ldx, const void *w, int ab_dtype,
                                   const float *bias, int64_t m, int64_t n, int64_t k, void *out, int64_t ldo,
                                   int out_dtype, int64_t norm_cols, const float *gamma, int64_t rope_cols,
                                   const float *rope_table) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, norm_cols >= 0 && norm_cols % 64 == 0 && norm_cols <= n && rope_cols >= 0 && rope_cols % 64 == 0 &&
                         rope_cols <= n,
                "p3d_linear_headnorm: norm/rope column counts must be multiples of the 64-wide head");
    P3D_REQUIRE(ctx, norm_cols == 0 || gamma, "p3d_linear_headnorm: gamma required");
    P3D_REQUIRE(ctx, rope_cols == 0 || rope_table, "p3d_linear_headnorm: rope table required");
    P3D_REQUIRE(ctx, n % 64 == 0, "p3d_linear_headnorm: n must be a multiple of 64");
    P3D_REQUIRE(ctx, norm_cols > 0 || rope_cols > 0, "p3d_linear_headnorm: nothing to fuse (use p3d_linear)");
    return linear_impl(ctx, x, ldx, w, ab_dtype, bias, m, n, k, out, ldo, out_dtype, P3D_EPI_NONE, nullptr, 0,
                       nullptr, 0, norm_cols, gamma, rope_cols, rope_table);
}

namespace {
int linear_impl(p3d_ctx *ctx, const void *x, int64_t ldx, const void *w, int ab_dtype, const float *bias, int64_t m,
                int64_t n, int64_t k, void *out, int64_t ldo, int out_dtype, int epilogue, const float *gate,
                int64_t gate_ld, const int32_t *batch_offsets, int nbatch, int64_t norm_cols, const float *norm_gamma,
                int64_t rope_cols, const float *rope) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && w && out, "p3d_linear: null pointer");
    P3D_REQUIRE(ctx, m >= 0 && n > 0 && k > 0, "p3d_linear: bad shape");
    P3D_REQUIRE(ctx, is_16bit(ab_dtype), "p3d_linear: operands must be bf16 or f16");
    P3D_REQUIRE(ctx, k % 8 == 0 && ldx % 8 == 0 && ldx >= k, "p3d_linear: k and ldx must be multiples of 8");
    P3D_REQUIRE(ctx, ldo >= n, "p3d_linear: ldo < n");
    P3D_REQUIRE(ctx, !(epilogue & P3D_EPI_RESIDUAL) || out_dtype == P3D_F32,
                "p3d_linear: residual epilogue needs f32 out");
    P3D_REQUIRE(ctx, !gate || (batch_offsets && nbatch > 0), "p3d_linear: gate needs batch offsets");
    if (m == 0) return P3D_OK;
    GemmParams p{};
    p.x = static_cast<const uint16_t *>(x);
    p.ldx = ldx;
    p.bias = bias;
    p.out = out;
    p.ldo = ldo;
    p.gate = gate;
    p.gate_ld = gate_ld;
    p.batch_offsets = batch_offsets;
    p.nbatch = nbatch;
    p.M = m;
    p.N = n;
    p.K = k;
    p.out_dtype = out_dtype;
    p.epi = epilogue;
    p.fault = ctx->fault;
    p.norm_cols = norm_cols;
    p.norm_gamma = norm_gamma;
    p.rope_cols = rope_cols;
    p.rope = reinterpret_cast<const float2 *>(rope);
    return run_gemm(ctx, x, ldx, w, ab_dtype, p);
}
}  // namespace

namespace p3d {
namespace {
// Bit t of tile_taps[b]: some row of rows [256 b, 256 b + 256) has a
// neighbour at tap t (nbr[t][row] in [0, n)).  One block per tile.
__global__ void __launch_bounds__(256) conv_tile_taps_kernel(const int32_t *__restrict__ nbr, int64_t n,
                                                             uint32_t *__restrict__ taps) {
    __shared__ uint32_t warp_or[8];
    const int64_t row = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
    uint32_t m = 0;
    if (row < n) {
#pragma unroll
        for (int t = 0; t < 27; ++t) {
            const int32_t s = __ldg(nbr + static_cast<int64_t>(t) * n + row);
            if (s >= 0 && s < n) m |= 1u << t;
        }
    }
    m = __reduce_or_sync(0xffffffffu, m);
    if ((threadIdx.x & 31) == 0) warp_or[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t r = 0;
        for (int i = 0; i < 8; ++i) r |= warp_or[i];
        taps[blockIdx.x] = r;
    }
}
}  // namespace
}  // namespace p3d

extern "C" int p3d_conv_tile_taps(p3d_ctx *ctx, const int32_t *nbr, int64_t n, uint32_t *tile_taps) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, nbr && tile_taps && n >= 0 && n < (int64_t(1) << 31), "p3d_conv_tile_taps: bad argument");
    if (n == 0) return P3D_OK;
    DeviceGuard guard(ctx->device);
    conv_tile_taps_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, ctx->stream>>>(nbr, n, tile_taps);
    return check_launch(ctx, "conv_tile_taps");
}

extern "C" int p3d_subm_conv3d(p3d_ctx *ctx, const void *x, int64_t n, int64_t cin, const int32_t *nbr,
                               const void *w, int ab_dtype, const float *bias, int64_t cout, void *out, int64_t ldo,
                               int out_dtype, int epilogue, const float *gate, int64_t gate_ld,
                               const int32_t *batch_offsets, int nbatch) {
    return p3d_subm_conv3d_taps(ctx, x, n, cin, nbr, w, ab_dtype, bias, cout, out, ldo, out_dtype, epilogue, gate,
                                gate_ld, batch_offsets, nbatch, nullptr);
}

extern "C" int p3d_subm_conv3d_taps(p3d_ctx *ctx, const void *x, int64_t n, int64_t cin, const int32_t *nbr,
                                    const void *w, int ab_dtype, const float *bias, int64_t cout, void *out,
                                    int64_t ldo, int out_dtype, int epilogue, const float *gate, int64_t gate_ld,
                                    const int32_t *batch_offsets, int nbatch, const uint32_t *tile_taps) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && nbr && w && out, "p3d_subm_conv3d: null pointer");
    P3D_REQUIRE(ctx, n >= 0 && cout > 0, "p3d_subm_conv3d: bad shape");
    P3D_REQUIRE(ctx, is_16bit(ab_dtype), "p3d_subm_conv3d: operands must be bf16 or f16");
    P3D_REQUIRE(ctx, cin % 64 == 0 && cin > 0, "p3d_subm_conv3d: cin must be a positive multiple of 64");
    P3D_REQUIRE(ctx, (reinterpret_cast<uintptr_t>(x) & 15) == 0, "p3d_subm_conv3d: x must be 16-byte aligned");
    P3D_REQUIRE(ctx, ldo >= cout, "p3d_subm_conv3d: ldo < cout");
    P3D_REQUIRE(ctx, !(epilogue & P3D_EPI_RESIDUAL) || out_dtype == P3D_F32,
                "p3d_subm_conv3d: residual epilogue needs f32 out");
    P3D_REQUIRE(ctx, !gate || (batch_offsets && nbatch > 0), "p3d_subm_conv3d: gate needs batch offsets");
    P3D_REQUIRE(ctx, n < (int64_t(1) << 31), "p3d_subm_conv3d: too many points");
    if (n == 0) return P3D_OK;
    // B operand: the 27 taps stacked as [27*cout, cin]; tap t occupies rows
    // [t*cout, (t+1)*cout), addressed in-kernel as row t*cout + n.
    GemmParams p{};
    p.x = static_cast<const uint16_t *>(x);
    p.ldx = cin;
    p.nbr = nbr;
    p.bias = bias;
    p.out = out;
    p.ldo = ldo;
    p.gate = gate;
    p.gate_ld = gate_ld;
    p.batch_offsets = batch_offsets;
    p.nbatch = nbatch;
    p.M = n;
    p.N = cout;
    p.K = cin;
    p.out_dtype = out_dtype;
    p.epi = epilogue;
    p.fault = ctx->fault;
    p.tile_taps = tile_taps;
    return run_gemm(ctx, nullptr, cin, w, ab_dtype, p);
}
