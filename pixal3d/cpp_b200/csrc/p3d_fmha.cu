// Varlen flash attention on tcgen05 tensor cores (head_dim 64).
//
// Replaces sparse_scaled_dot_product_attention (src/sparse.cpp:704-783) and
// sparse_cross_attention (src/sparse.cpp:785-859): sequence s attends query
// rows [cu_q[s], cu_q[s+1]) to key/value rows [cu_k[s], cu_k[s+1]).  The
// reference's two-pass softmax becomes an online softmax (f32 running max
// and sum, logits pre-scaled by log2(e)); scores never leave the SM.
//
// One CTA = 128 query rows of one head; two CTAs share an SM (256 TMEM
// columns each) so one CTA's softmax overlaps the other's tensor-core work.
// 6 warps:
//   warp 0     TMA producer: Q once, then K/V blocks of 64 keys (3 stages)
//   warp 1     TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2-5  softmax: thread = query row = TMEM lane (warp w reads lane
//              quarter w % 4)
// Per key block j (S/P buffer b = j & 1 in TMEM):
//   S_b = Q K_j^T              tcgen05.mma, A = Q (smem), B = K (smem), K-major
//   P_b = exp2(S_b*c - m)      softmax threads: tcgen05.ld S row, exponents in
//                              packed 16-bit pairs (ex2.approx.f16x2 /
//                              .bf16x2: two per MUFU op), written as P back
//                              into S_b's columns
//   O  += P_b V_j              tcgen05.mma with A read from TMEM (P_b),
//                              B = V (smem, MN-major); O stays in TMEM
//   l  += P_b 1                the row sums, by the tensor core from the same
//                              16-bit P: the P V MMA has N = 80, its last 16
//                              columns reading a ones tile (l = O column 64)
// The running max m is raised lazily: only when a block's max exceeds it by
// more than 8 (a factor 2^8 in P) does the row's owner wait for the pending
// P V, rescale O and l in TMEM (ld, scale, st); otherwise P is computed
// against the stale max, which is exact because the final normalisation
// divides by a sum taken against the same max.
// Every mbarrier wait is bounded; a stuck pipeline latches P3D_ERR_TIMEOUT,
// the CTA still frees its TMEM and exits.
#include <type_traits>

#include "p3d_common.cuh"

namespace p3d {
namespace {

constexpr int kM = 128;       // query rows per CTA
constexpr int kN = 64;        // keys per block
constexpr int kD = 64;        // head dim
constexpr int kStages = 3;    // K/V stages
constexpr int kThreadsF = 192;
constexpr float kRescaleLog2 = 8.0f;

constexpr int Q_BYTES = kM * kD * 2;   // 16 KB
constexpr int KV_BYTES = kN * kD * 2;  // 8 KB each
// Ones companion of the V stages: the P V MMA runs with N = 80 (64 value
// dims + 16 ones columns), its second 64-wide MN group read kStages * KV_BYTES
// past each V stage, so the accumulator's columns 64..79 receive the row sums
// of the same 16-bit P.
constexpr int ONES_BYTES = kStages * KV_BYTES;
constexpr int USED_BYTES = Q_BYTES + kStages * 2 * KV_BYTES + ONES_BYTES + 1024 + 512;
// Request enough dynamic shared memory that at most two CTAs fit on an SM:
// two CTAs use 2 x 256 = 512 TMEM columns, a third would wait in tcgen05.alloc.
constexpr int SMEM_BYTES = 100 * 1024;
static_assert(USED_BYTES <= SMEM_BYTES, "smem layout exceeds the request");
constexpr uint32_t TMEM_COLS = 256;  // S/P 0 (64) | S/P 1 (64) | O (64) | l (16) | unused
constexpr uint32_t O_COL = 128;
constexpr uint32_t L_COL = 192;
static_assert(L_COL == O_COL + kD, "the row sum is accumulator column 64 of the N = 80 P V MMA");

__device__ __forceinline__ uint32_t sp_col(int b) { return b ? 64u : 0u; }

// D(tmem) (+)= A(tmem) * B(smem desc)^T, kind::f16.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// One TMEM column for the warp's 32 lanes.
__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
    uint32_t r;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr) : "memory");
    return __uint_as_float(r);
}
__device__ __forceinline__ void tmem_st1(uint32_t taddr, float v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(__float_as_uint(v))
                 : "memory");
}

// 2^x0, 2^x1 as a packed 16-bit pair (x0 in the low half): one MUFU op.
template <typename T>
__device__ __forceinline__ uint32_t ex2_pair(float x0, float x1);
template <>
__device__ __forceinline__ uint32_t ex2_pair<__half>(float x0, float x1) {
    uint32_t r;
    asm("{\n\t.reg .b32 t;\n\tcvt.rn.f16x2.f32 t, %2, %1;\n\tex2.approx.f16x2 %0, t;\n\t}"
        : "=r"(r)
        : "f"(x0), "f"(x1));
    return r;
}
template <>
__device__ __forceinline__ uint32_t ex2_pair<__nv_bfloat16>(float x0, float x1) {
    uint32_t r;
    asm("{\n\t.reg .b32 t;\n\tcvt.rn.bf16x2.f32 t, %2, %1;\n\tex2.approx.ftz.bf16x2 %0, t;\n\t}"
        : "=r"(r)
        : "f"(x0), "f"(x1));
    return r;
}

// (a0, a1) * s + (c, c) as one packed f32x2 FMA.
__device__ __forceinline__ void ffma2(float a0, float a1, float s, float c, float &d0, float &d1) {
    unsigned long long a, sc, cc, d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %1};" : "=l"(sc) : "f"(s));
    asm("mov.b64 %0, {%1, %1};" : "=l"(cc) : "f"(c));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(sc), "l"(cc));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Row max of 64 scores: 8 chains of 3-input max, then a 3-input tree.
__device__ __forceinline__ float row_max64(const float *s) {
    float m[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float a = max3f(s[c], s[8 + c], s[16 + c]);
        const float b = max3f(a, s[24 + c], s[32 + c]);
        const float d = max3f(b, s[40 + c], s[48 + c]);
        m[c] = fmaxf(d, s[56 + c]);
    }
    return max3f(max3f(m[0], m[1], m[2]), max3f(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
}

// P for 64 scores: x = s * scale_log2 - m by packed f32x2 FMAs, 2^x in
// packed 16-bit pairs on MUFU.  (Computing part of the exponentials on the
// FMA pipe by a polynomial measured slower here: the softmax warps are bound
// by FMA-pipe issue, not by MUFU.)
template <typename T>
__device__ __forceinline__ void softmax_p64(const float *s, float scale_log2, float nm, uint32_t (&pk)[32]) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        float x0, x1;
        ffma2(s[2 * i], s[2 * i + 1], scale_log2, nm, x0, x1);
        pk[i] = ex2_pair<T>(x0, x1);
    }
}

struct FmhaParams {
    const int32_t *cu_q, *cu_k;
    void *out;
    int64_t ldo;
    float scale_log2;
    int *fault;
};

template <typename T>
__global__ void __launch_bounds__(kThreadsF, 2)
    fmha_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const FmhaParams p) {
    pdl_wait();  // q/k/v and the sequence offsets come from the previous kernels
    pdl_trigger();
    const int seq = blockIdx.z, head = blockIdx.y;
    const int q0 = p.cu_q[seq], q1 = p.cu_q[seq + 1];
    const int k0 = p.cu_k[seq], k1 = p.cu_k[seq + 1];
    const int qt = q0 + blockIdx.x * kM;
    if (qt >= q1 || k1 <= k0) return;
    const int nblk = (k1 - k0 + kN - 1) / kN;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *sQ = smem;
    uint8_t *sK = sQ + Q_BYTES;             // [kStages][KV_BYTES]
    uint8_t *sV = sK + kStages * KV_BYTES;  // [kStages][KV_BYTES]
    uint8_t *sOnes = sV + kStages * KV_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sOnes + ONES_BYTES);
    uint64_t *q_full = bars;                 // 1
    uint64_t *kv_full = bars + 1;            // kStages
    uint64_t *kv_empty = kv_full + kStages;  // kStages
    uint64_t *s_full = kv_empty + kStages;   // 2
    uint64_t *p_full = s_full + 2;           // 2
    uint64_t *pv_done = p_full + 2;          // 2
    uint64_t *done_bar = pv_done + 2;        // 1
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done_bar + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], 4);
            mbar_init(&pv_done[b], 1);
        }
        mbar_init(done_bar, 1);
        fence_barrier_init();
        prefetch_tmap(&tq);
        prefetch_tmap(&tk);
        prefetch_tmap(&tv);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    {
        // ones tile (16-bit 1.0) for the row-sum MMA; read by the async proxy
        const uint32_t one2 = std::is_same<T, __nv_bfloat16>::value ? 0x3F803F80u : 0x3C003C00u;
        uint32_t *o32 = reinterpret_cast<uint32_t *>(sOnes);
        for (int i = threadIdx.x; i < ONES_BYTES / 4; i += kThreadsF) o32[i] = one2;
        fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;

    if (warp == 0) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, Q_BYTES);
            tma_load_2d(sQ, &tq, q_full, head * kD, qt);
            int stage = 0;
            uint32_t phase = 0;
            for (int j = 0; j < nblk; ++j) {
                if (!mbar_wait(&kv_empty[stage], phase ^ 1, p.fault)) break;
                mbar_arrive_expect_tx(&kv_full[stage], 2 * KV_BYTES);
                tma_load_2d(sK + stage * KV_BYTES, &tk, &kv_full[stage], head * kD, k0 + j * kN);
                tma_load_2d(sV + stage * KV_BYTES, &tv, &kv_full[stage], head * kD, k0 + j * kN);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA
        if (lane == 0) {
            const uint32_t idesc_s = idesc_f32acc(kM, kN, kBf16);
            const uint32_t idesc_ol = idesc_f32acc(kM, kD + 16, kBf16, true);  // O and l together
            const uint32_t q_addr = smem_u32(sQ);
            bool ok = mbar_wait(q_full, 0, p.fault);
            auto issue_pv = [&](int i) -> bool {
                const int b = i & 1, st = i % kStages;
                if (!mbar_wait(&p_full[b], (i >> 1) & 1, p.fault)) return false;
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sV + st * KV_BYTES);
#pragma unroll
                for (int kk = 0; kk < kN / 16; ++kk)  // 16 keys = 8 packed TMEM columns of P
                    umma_f16_ts(tmem + O_COL, tmem + sp_col(b) + kk * 8,
                                sw128_desc_mn(v_addr + kk * 2048, kStages * KV_BYTES), idesc_ol,
                                (i > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&pv_done[b]);
                umma_commit(&kv_empty[st]);
                return true;
            };
            for (int j = 0; j < nblk && ok; ++j) {
                const int b = j & 1, st = j % kStages;
                if (!mbar_wait(&kv_full[st], (j / kStages) & 1, p.fault)) { ok = false; break; }
                // S/P buffer b was last read by P(j-2) V(j-2)
                if (j >= 2 && !mbar_wait(&pv_done[b], ((j - 2) >> 1) & 1, p.fault)) { ok = false; break; }
                tc_fence_after();
                const uint32_t k_addr = smem_u32(sK + st * KV_BYTES);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk)
                    umma_f16(tmem + sp_col(b), sw128_desc(q_addr + kk * 32), sw128_desc(k_addr + kk * 32), idesc_s,
                             kk > 0 ? 1u : 0u);
                umma_commit(&s_full[b]);
                if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
            }
            if (ok) issue_pv(nblk - 1);
            umma_commit(done_bar);
            mbar_wait(done_bar, 0, p.fault);
        }
        __syncwarp();
    } else {
        // --------------------------------------------------------- softmax
        const int q = warp & 3;  // TMEM lane quarter
        const int row = q * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        float m_run = -INFINITY;
        bool ok = true;
        // Waits are warp-uniform (lane 0 polls) because the tcgen05.ld/st
        // that follow are warp-collective.
        auto warp_wait = [&](uint64_t *bar, uint32_t parity) -> bool {
            int r = 1;
            if (lane == 0) r = mbar_wait(bar, parity, p.fault) ? 1 : 0;
            return __shfl_sync(0xffffffffu, r, 0) != 0;
        };
        for (int j = 0; j < nblk && ok; ++j) {
            const int b = j & 1;
            if (!warp_wait(&s_full[b], (j >> 1) & 1)) { ok = false; break; }
            tc_fence_after();
            float s[kN];
            {
                float v0[32], v1[32];
                tmem_ld32(tmem + lane_base + sp_col(b), v0);
                tmem_ld32(tmem + lane_base + sp_col(b) + 32, v1);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    s[i] = v0[i];
                    s[32 + i] = v1[i];
                }
            }
            const int valid = min(kN, k1 - (k0 + j * kN));
            if (valid < kN) {
#pragma unroll
                for (int i = 0; i < kN; ++i) s[i] = i < valid ? s[i] : -INFINITY;
            }
            float mx = row_max64(s) * p.scale_log2;
            const bool need = j > 0 && mx > m_run + kRescaleLog2;
            if (j == 0) m_run = mx;
            if (__any_sync(0xffffffffu, need)) {
                // raise the running max of the rows that need it: O (after the
                // pending P V) and l scale by 2^(m_old - m_new); other rows of
                // the warp take part with a factor of 1.
                if (!warp_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1)) { ok = false; break; }
                tc_fence_after();
                const float alpha = need ? exp2f(m_run - mx) : 1.0f;
                if (need) m_run = mx;
#pragma unroll
                for (int c = 0; c < kD; c += 32) {
                    float o[32];
                    tmem_ld32(tmem + lane_base + O_COL + c, o);
                    tmem_ld_wait();
                    uint32_t r[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(o[i] * alpha);
                    tmem_st32(tmem + lane_base + O_COL + c, r);
                }
                const float l = tmem_ld1(tmem + lane_base + L_COL);
                tmem_ld_wait();
                tmem_st1(tmem + lane_base + L_COL, l * alpha);
                tmem_st_wait();
            }
            uint32_t pk[32];
            softmax_p64<T>(s, p.scale_log2, -m_run, pk);
            tmem_st32(tmem + lane_base + sp_col(b), pk);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[b]);
        }
        // all P V done -> normalise O and store this row (64 dims, 128 bytes)
        if (ok) ok = warp_wait(&pv_done[(nblk - 1) & 1], ((nblk - 1) >> 1) & 1);
        tc_fence_after();
        const int64_t grow = static_cast<int64_t>(qt) + row;
        float o[kD];
#pragma unroll
        for (int c = 0; c < kD; c += 32) {
            float v[32];
            tmem_ld32(tmem + lane_base + O_COL + c, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[c + i] = v[i];
        }
        const float l_run = tmem_ld1(tmem + lane_base + L_COL);
        tmem_ld_wait();
        if (ok && grow < q1) {
            const float inv = 1.0f / l_run;
            T *dst = reinterpret_cast<T *>(p.out) + grow * p.ldo + head * kD;
#pragma unroll
            for (int c = 0; c < kD; c += 8) {
                uint4 u;
                u.x = pack2<T>(o[c] * inv, o[c + 1] * inv);
                u.y = pack2<T>(o[c + 2] * inv, o[c + 3] * inv);
                u.z = pack2<T>(o[c + 4] * inv, o[c + 5] * inv);
                u.w = pack2<T>(o[c + 6] * inv, o[c + 7] * inv);
                *reinterpret_cast<uint4 *>(dst + c) = u;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace
}  // namespace p3d

using namespace p3d;

// Launch for head_dim 64 (called by the attention entry points).
int p3d_fmha_tc(p3d_ctx *ctx, const void *q, int64_t ldq, const void *k, int64_t ldk, const void *v, int64_t ldv,
                void *out, int64_t ldo, const int32_t *cu_q, const int32_t *cu_k, int nseq, int64_t max_q,
                int64_t rows_q, int64_t rows_k, int heads, float scale, int dtype) {
    // Tensor maps over the whole q / k / v views: rows x (heads*64) columns,
    // boxes of 64 columns (one head) x 128 (Q) or 64 (K, V) rows, 128B swizzle.
    CUtensorMap tq, tk, tv;
    int rc = make_tmap_16bit_2d(ctx, &tq, q, dtype, rows_q, static_cast<uint64_t>(heads) * kD, ldq, kM);
    if (rc) return rc;
    rc = make_tmap_16bit_2d(ctx, &tk, k, dtype, rows_k, static_cast<uint64_t>(heads) * kD, ldk, kN);
    if (rc) return rc;
    rc = make_tmap_16bit_2d(ctx, &tv, v, dtype, rows_k, static_cast<uint64_t>(heads) * kD, ldv, kN);
    if (rc) return rc;
    FmhaParams p{};
    p.cu_q = cu_q;
    p.cu_k = cu_k;
    p.out = out;
    p.ldo = ldo;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.fault = ctx->fault;
    static bool attr_done[2] = {false, false};
    dim3 grid(static_cast<unsigned>(ceil_div(max_q, kM)), heads, nseq);
    if (dtype == P3D_BF16) {
        if (!attr_done[0]) {
            P3D_CUDA(ctx, cudaFuncSetAttribute(fmha_tc_kernel<__nv_bfloat16>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
            attr_done[0] = true;
        }
        P3D_CUDA(ctx, launch_pdl(fmha_tc_kernel<__nv_bfloat16>, grid, dim3(kThreadsF), SMEM_BYTES, ctx->stream, tq, tk,
                                 tv, p));
    } else {
        if (!attr_done[1]) {
            P3D_CUDA(ctx, cudaFuncSetAttribute(fmha_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               SMEM_BYTES));
            attr_done[1] = true;
        }
        P3D_CUDA(ctx, launch_pdl(fmha_tc_kernel<__half>, grid, dim3(kThreadsF), SMEM_BYTES, ctx->stream, tq, tk, tv, p));
    }
    return check_launch(ctx, "fmha_tc");
}
