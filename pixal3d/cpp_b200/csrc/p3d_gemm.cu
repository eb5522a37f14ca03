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
// CTA = 9 warps, one CTA per SM, persistent over output tiles (n fastest so
// concurrently running CTAs share A tiles through L2):
//   warps 0-3  producers: thread 0 issues TMA; for the gather variant all
//              128 threads issue the row gathers (cp.async, 8 x 16 B each)
//   warps 4-7  epilogue: tcgen05.ld 32 lanes x 32 columns per warp, bias /
//              activation / gated residual, vector stores
//   warp  8    TMEM allocator + single-thread tcgen05.mma issuer
// Tile 128 x BN (BN in {64,128,256}), BK = 64 (one 128-byte swizzle atom),
// UMMA 128 x BN x 16; accumulators double-buffered in TMEM (2*BN columns) so
// the epilogue of tile i overlaps the main loop of tile i+1.
// Every mbarrier wait is bounded (p3d_common.cuh): a stuck pipeline latches
// P3D_ERR_TIMEOUT and the kernel still frees its TMEM and exits.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "p3d_common.cuh"

namespace p3d {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kProducerThreads = 128;
constexpr int kThreads = 9 * 32;
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
    // [0, rope_cols) are then rotated with rope[row][pair] = (cos, sin).
    int64_t norm_cols, rope_cols;
    const float *norm_gamma;
    const float2 *rope;
};

// MT = 128-row M sub-tiles per CTA tile; they share every B stage, which
// halves the B operand stream per FLOP when MT = 2.
template <int BN, int MT>
struct Cfg {
    static constexpr int A_BYTES = MT * BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (196608 / STAGE_BYTES) > 8 ? 8 : (196608 / STAGE_BYTES);
    static constexpr int ACC_COLS = MT * BN;                 // one accumulator buffer
    static constexpr int ACC_BUFS = 2 * ACC_COLS <= 512 ? 2 : 1;
    static constexpr int TMEM_COLS = ACC_BUFS * ACC_COLS <= 128 ? 128 : (ACC_BUFS * ACC_COLS <= 256 ? 256 : 512);
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
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

template <int BN, bool GATHER, int MT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const GemmParams p) {
    using C = Cfg<BN, MT>;
    constexpr int BMT = BM * MT;  // rows per CTA tile
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint8_t *smem_a = smem;
    uint8_t *smem_b = smem + STAGES * C::A_BYTES;
    uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem_b + STAGES * C::B_BYTES);
    uint64_t *empty_bar = full_bar + STAGES;
    uint64_t *tfull_bar = empty_bar + STAGES;  // [2]
    uint64_t *tempty_bar = tfull_bar + 2;      // [2]
    uint64_t *done_bar = tempty_bar + 2;       // [1]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done_bar + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    const int64_t m_tiles = (p.M + BMT - 1) / BMT;
    const int64_t n_tiles = (p.N + BN - 1) / BN;
    const int64_t num_tiles = m_tiles * n_tiles;
    const int kblocks_per_tap = static_cast<int>((p.K + BK - 1) / BK);
    const int num_kb = GATHER ? 27 * kblocks_per_tap : kblocks_per_tap;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], GATHER ? (kProducerThreads + 1) : 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], 4);
        }
        mbar_init(done_bar, 1);
        fence_barrier_init();
        if (!GATHER) prefetch_tmap(&tmap_a);
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

    if (warp < 4) {
        // ------------------------------------------------------------ producer
        const int t = threadIdx.x;  // 0..127
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int64_t tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
            const int64_t m0 = (tile / n_tiles) * BMT;
            const int64_t n0 = (tile % n_tiles) * BN;
            for (int kb = 0; kb < num_kb; ++kb) {
                if (GATHER) {
                    // warp-uniform bounded wait (lane 0 polls, the warp follows)
                    int w_ok = 1;
                    if ((t & 31) == 0) w_ok = mbar_wait(&empty_bar[stage], phase ^ 1, p.fault) ? 1 : 0;
                    if (!__shfl_sync(0xffffffffu, w_ok, 0)) {
                        ok = false;
                        break;
                    }
                } else if (t == 0) {
                    if (!mbar_wait(&empty_bar[stage], phase ^ 1, p.fault)) {
                        ok = false;
                        break;
                    }
                }
                uint8_t *sa = smem_a + stage * C::A_BYTES;
                uint8_t *sb = smem_b + stage * C::B_BYTES;
                if (GATHER) {
                    const int tap = kb / kblocks_per_tap;
                    const int kc = (kb % kblocks_per_tap) * BK;
                    // Warp w owns tile rows [w*32*MT, (w+1)*32*MT).  Per 32-row
                    // slice, lane l fetches the source row of slice row l;
                    // each cp.async instruction then copies 4 whole rows, 8
                    // lanes per 128-byte row: coalesced global reads and
                    // conflict-free swizzled shared-memory writes.
                    const int lane_ = t & 31;
                    const int chunk = lane_ & 7;
#pragma unroll
                    for (int sl = 0; sl < MT; ++sl) {
                        const int wrow0 = ((t >> 5) * MT + sl) * 32;
                        const int64_t row = m0 + wrow0 + lane_;
                        int32_t my_src = -1;
                        if (row < p.M) {
                            my_src = __ldg(p.nbr + static_cast<int64_t>(tap) * p.M + row);
                            if (my_src >= p.M || my_src < 0) my_src = -1;  // sentinel -> zero row
                        }
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int r = wrow0 + i * 4 + (lane_ >> 3);
                            const int32_t src = __shfl_sync(0xffffffffu, my_src, i * 4 + (lane_ >> 3));
                            const uint16_t *g =
                                p.x + (src >= 0 ? static_cast<int64_t>(src) * p.ldx + kc + chunk * 8 : 0);
                            cp_async16(sa + r * 128 + ((chunk ^ (r & 7)) << 4), g, src >= 0 ? 16u : 0u);
                        }
                    }
                    if (t == 0) {
                        mbar_arrive_expect_tx(&full_bar[stage], C::B_BYTES);
                        // Tap t's weights are rows [t*N, (t+1)*N) of the stacked [27*N, K] map.
                        tma_load_2d(sb, &tmap_b, &full_bar[stage], kc, static_cast<int>(tap * p.N + n0));
                    }
                    cp_async_mbar_arrive_noinc(&full_bar[stage]);
                } else if (t == 0) {
                    mbar_arrive_expect_tx(&full_bar[stage], C::A_BYTES + C::B_BYTES);
#pragma unroll
                    for (int sl = 0; sl < MT; ++sl)
                        tma_load_2d(sa + sl * (BM * 128), &tmap_a, &full_bar[stage], kb * BK,
                                    static_cast<int>(m0 + sl * BM));
                    tma_load_2d(sb, &tmap_b, &full_bar[stage], kb * BK, static_cast<int>(n0));
                }
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
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
            for (int64_t tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, p.fault)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * C::ACC_COLS;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&full_bar[stage], phase, p.fault)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (GATHER) fence_proxy_async_smem();
                    const uint32_t a_addr = smem_u32(smem_a + stage * C::A_BYTES);
                    const uint32_t b_addr = smem_u32(smem_b + stage * C::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
                        for (int sl = 0; sl < MT; ++sl)
                            umma_f16(d_tmem + sl * BN, sw128_desc(a_addr + sl * (BM * 128) + kk * 32),
                                     sw128_desc(b_addr + kk * 32), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    }
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
    } else {
        // ----------------------------------------------------------- epilogue
        const int q = warp & 3;  // TMEM lane quarter accessible to this warp
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int64_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            const int64_t m0 = (tile / n_tiles) * BMT;
            const int64_t n0 = (tile % n_tiles) * BN;
            if (!mbar_wait(&tfull_bar[acc], acc_phase, p.fault)) break;
            tc_fence_after();
            if (p.norm_cols > 0 || p.rope_cols > 0) {
                // 64-column groups = one head: bias, per-head RMS norm with gamma,
                // interleaved RoPE from the per-row cos/sin table, then store.
#pragma unroll 1
                for (int cs = 0; cs < MT * BN; cs += 64) {
                    const int sl = cs / BN, c0 = cs % BN;
                    const int64_t row = m0 + sl * BM + q * 32 + lane;
                    float v[64];
                    {
                        float a[32], b[32];
                        const uint32_t ta = tmem_base + acc * C::ACC_COLS + cs + (static_cast<uint32_t>(q * 32) << 16);
                        tmem_ld32(ta, a);
                        tmem_ld32(ta + 32, b);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            v[i] = a[i];
                            v[32 + i] = b[i];
                        }
                    }
                    const int64_t col0 = n0 + c0;
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
                            const float2 *cs2 = p.rope + row * 32;
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                const float2 r = __ldg(cs2 + i);
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
            } else {
#pragma unroll 1
            for (int cs = 0; cs < MT * BN; cs += 32) {
                const int sl = cs / BN, c0 = cs % BN;
                const int64_t row = m0 + sl * BM + q * 32 + lane;
                float v[32];
                tmem_ld32(tmem_base + acc * C::ACC_COLS + cs + (static_cast<uint32_t>(q * 32) << 16), v);
                tmem_ld_wait();
                const int64_t col0 = n0 + c0;
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
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty_bar[acc]);
            if (++acc == C::ACC_BUFS) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) tmem_dealloc(tmem_base, C::TMEM_COLS);
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

template <int BN, bool GATHER, int MT>
int launch_gemm(p3d_ctx *ctx, const CUtensorMap &ta, const CUtensorMap &tb, const GemmParams &p) {
    using C = Cfg<BN, MT>;
    static bool attr_set = false;
    if (!attr_set) {
        P3D_CUDA(ctx, cudaFuncSetAttribute(gemm_tc_kernel<BN, GATHER, MT>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr_set = true;
    }
    const int64_t tiles = ceil_div(p.M, BM * MT) * ceil_div(p.N, BN);
    const int grid = static_cast<int>(std::min<int64_t>(tiles, ctx->num_sms));
    gemm_tc_kernel<BN, GATHER, MT><<<grid, kThreads, C::SMEM, ctx->stream>>>(ta, tb, p);
    return check_launch(ctx, "gemm_tc_kernel");
}

int pick_bn(int64_t n) {
    if (n <= 64) return 64;
    if (n <= 128) return 128;
    return 256;
}

int run_gemm(p3d_ctx *ctx, const CUtensorMap *ta, const CUtensorMap &tb, const GemmParams &p, bool gather) {
    const int bn = pick_bn(p.N);
    CUtensorMap dummy = tb;
    const CUtensorMap &a = ta ? *ta : dummy;
    if (gather) {
        // Long K loops (27 taps x Cin/64): two 128-row sub-tiles per CTA share
        // every B stage once there are enough 256-row tiles to fill the GPU.
        // Measured on B200: MT = 2 (3 stages) is slower than MT = 1 (4 stages) for
        // the config-2 conv (3.13 vs 2.55 ms), so the gather path uses MT = 1.
        const bool mt2 = false;
        if (bn == 64) return mt2 ? launch_gemm<64, true, 2>(ctx, a, tb, p) : launch_gemm<64, true, 1>(ctx, a, tb, p);
        if (bn == 128) return mt2 ? launch_gemm<128, true, 2>(ctx, a, tb, p) : launch_gemm<128, true, 1>(ctx, a, tb, p);
        return mt2 ? launch_gemm<256, true, 2>(ctx, a, tb, p) : launch_gemm<256, true, 1>(ctx, a, tb, p);
    }
    if (bn == 64) return launch_gemm<64, false, 1>(ctx, a, tb, p);
    if (bn == 128) return launch_gemm<128, false, 1>(ctx, a, tb, p);
    return launch_gemm<256, false, 1>(ctx, a, tb, p);
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
    const int bn = pick_bn(n);
    CUtensorMap ta, tb;
    int rc = make_tmap_16bit_2d(ctx, &ta, x, ab_dtype, m, k, ldx, BM);
    if (rc) return rc;
    rc = make_tmap_16bit_2d(ctx, &tb, w, ab_dtype, n, k, k, bn);
    if (rc) return rc;
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
    p.idesc = idesc_f32acc(BM, bn, ab_dtype == P3D_BF16);
    p.epi = epilogue;
    p.fault = ctx->fault;
    p.norm_cols = norm_cols;
    p.norm_gamma = norm_gamma;
    p.rope_cols = rope_cols;
    p.rope = reinterpret_cast<const float2 *>(rope);
    return run_gemm(ctx, &ta, tb, p, false);
}
}  // namespace

extern "C" int p3d_subm_conv3d(p3d_ctx *ctx, const void *x, int64_t n, int64_t cin, const int32_t *nbr,
                               const void *w, int ab_dtype, const float *bias, int64_t cout, void *out, int64_t ldo,
                               int out_dtype, int epilogue, const float *gate, int64_t gate_ld,
                               const int32_t *batch_offsets, int nbatch) {
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
    const int bn = pick_bn(cout);
    // B operand: the 27 taps stacked as [27*cout, cin]; tap t occupies rows
    // [t*cout, (t+1)*cout).  The kernel addresses tap t with row coordinate
    // n0 + t*cout through a per-tap map, so encode one map per launch over
    // the whole stack and offset rows in-kernel.
    CUtensorMap tb;
    int rc = make_tmap_16bit_2d(ctx, &tb, w, ab_dtype, 27 * cout, cin, cin, bn);
    if (rc) return rc;
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
    p.idesc = idesc_f32acc(BM, bn, ab_dtype == P3D_BF16);
    p.epi = epilogue;
    p.fault = ctx->fault;
    return run_gemm(ctx, nullptr, tb, p, true);
}
