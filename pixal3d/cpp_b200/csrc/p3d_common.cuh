// Shared device/host helpers for the sm_100a SLat kernels.
//
// - p3d_ctx: device, stream, error message, device fault latch.
// - Bounded waits: every spin on an mbarrier gives up after a wall-clock
//   limit (globaltimer), latches P3D_ERR_TIMEOUT in the device flag and
//   returns false, so a broken pipeline ends the kernel instead of hanging
//   the GPU.
// - Thin inline-PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor, no
//   multicast), cp.async, tcgen05 (alloc/mma/commit/ld/fence).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "p3d.h"

struct p3d_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    int num_sms = 148;
    int *fault = nullptr;  // device flag: first latched p3d_status
    std::string error;
    int64_t launches = 0;
};

namespace p3d {

// ----------------------------------------------------------------- host side

int set_error(p3d_ctx *ctx, int status, const std::string &msg);
int check_launch(p3d_ctx *ctx, const char *what);

// ---- Programmatic dependent launch.  A kernel launched by launch_pdl may
// start (its prologue: barrier init, TMEM allocation, tensor-map prefetch)
// while the previous kernel in the stream is still running; it must call
// pdl_wait() before its first access to global memory another kernel wrote or
// reads (the wait returns once the previous grid has completed and its writes
// are visible; without a programmatic dependency it returns at once).
// pdl_trigger() lets the next such kernel be scheduled once every CTA of this
// grid has triggered or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Makes `device` current for the guard's scope and restores the caller's.
struct DeviceGuard {
    int prev = -1;
    bool switched = false;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != device && cudaSetDevice(device) == cudaSuccess)
            switched = true;
    }
    ~DeviceGuard() {
        if (switched) cudaSetDevice(prev);
    }
};

#define P3D_REQUIRE(ctx, cond, msg)                                                   \
    do {                                                                              \
        if (!(cond)) return ::p3d::set_error((ctx), P3D_ERR_INVALID, (msg));          \
    } while (0)

#define P3D_CUDA(ctx, expr)                                                           \
    do {                                                                              \
        cudaError_t e_ = (expr);                                                      \
        if (e_ != cudaSuccess)                                                        \
            return ::p3d::set_error((ctx), P3D_ERR_CUDA,                              \
                                    std::string(#expr ": ") + cudaGetErrorString(e_)); \
    } while (0)

// Encode a 2D 16-bit (bf16/f16) tensor map (rows x cols, row pitch in elements) with a
// box of box_rows x 64 columns and 128-byte swizzle, the canonical K-major
// SW128 operand layout of tcgen05.mma.
int make_tmap_16bit_2d(p3d_ctx *ctx, CUtensorMap *map, const void *base, int dtype, uint64_t rows, uint64_t cols,
                       uint64_t pitch_elems, uint32_t box_rows);

// ---------------------------------------------------------------- device side

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per wait

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void latch_fault(int *fault, int status) {
    if (fault) atomicCAS(fault, 0, status);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: true when the phase completed, false once limit_ns passed
// without it (P3D_ERR_TIMEOUT latched in *fault).  Every pipeline wait of the
// library goes through this routine with kWaitLimitNs; p3d_wait_selftest
// drives it to expiry with a short limit.
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, uint32_t parity, int *fault, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer() - t0 > limit_ns) {
            latch_fault(fault, P3D_ERR_TIMEOUT);
            return false;
        }
    }
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *fault) {
    return mbar_wait_for(bar, parity, fault, kWaitLimitNs);
}
// Arrive on `bar` when all cp.async issued so far by this thread complete.
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---- cp.async (16-byte, zero-fill when src_bytes == 0)
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- TMA (tiled 2D load, no multicast)
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
// TMA row gather: 4 rows (row0..row3) x box-width columns starting at column
// c0, box one row high, written as 4 consecutive box rows at smem_dst.  A row
// index outside the tensor reads the fill value (zero).  No multicast.
__device__ __forceinline__ void tma_gather4(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int c0, int r0,
                                            int r1, int r2, int r3) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4, %5, %6, %7}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(r0), "r"(r1), "r"(r2), "r"(r3)
        : "memory");
}
// tma_gather4 into this CTA's shared memory with the completion counted on
// the mbarrier at a shared::cluster address (the even CTA's, in a CTA pair).
// No multicast.
__device__ __forceinline__ void tma_gather4_pair(void *smem_dst, const CUtensorMap *map, uint32_t bar_cluster_addr,
                                                 int c0, int r0, int r1, int r2, int r3) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], "
        "[%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(r0), "r"(r1), "r"(r2), "r"(r3)
        : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (bf16/f16 in, f32 acc).
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on an mbarrier when all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
// ---- 2-CTA (cluster pair) forms: cta_group::2 MMA over both SMs' shared
// memory, accumulators in both SMs' TMEM.  No TMA multicast is used.
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait with cluster-scope acquire (arrivals may come from the peer CTA).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, int *fault) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (globaltimer() - t0 > kWaitLimitNs) {
            latch_fault(fault, P3D_ERR_TIMEOUT);
            return false;
        }
    }
}
__device__ __forceinline__ void tmem_alloc2(uint32_t *smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// TMA 2D tile load into this CTA's shared memory whose completion is counted
// on an mbarrier of either CTA of the pair (cluster address), e.g. the even
// CTA's.  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const CUtensorMap *map, uint32_t bar_cluster_addr,
                                                 int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
        : "memory");
}
// Pair MMA issued by the even CTA: A rows [0,128) from each CTA's own shared
// memory (M = 256), B's N/2 halves from each CTA, D in each CTA's TMEM.
__device__ __forceinline__ void umma2_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on the mbarrier at a shared::cluster address (this CTA's or the
// peer's) when all pair MMAs issued so far by this thread complete.
__device__ __forceinline__ void umma_commit2(uint32_t cluster_addr) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Wait for this thread's tcgen05.ld results and tie the 32 registers to the
// wait, so no use of them is scheduled above it.
__device__ __forceinline__ void tmem_ld_wait_regs(float (&v)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7]),
                   "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]), "+f"(v[12]), "+f"(v[13]), "+f"(v[14]),
                   "+f"(v[15]), "+f"(v[16]), "+f"(v[17]), "+f"(v[18]), "+f"(v[19]), "+f"(v[20]), "+f"(v[21]),
                   "+f"(v[22]), "+f"(v[23]), "+f"(v[24]), "+f"(v[25]), "+f"(v[26]), "+f"(v[27]), "+f"(v[28]),
                   "+f"(v[29]), "+f"(v[30]), "+f"(v[31])
                 :
                 : "memory");
}

// ---- TMA store / reduce-add from shared memory (bulk async-group completion)
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *smem_src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
                 : "memory");
}
// global[tile] += shared tile (element type of the map; f32 here), performed
// by the TMA unit at L2: a residual add without reading the residual into the SM.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, const void *smem_src, int c0, int c1) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// At most N of this thread's bulk groups still reading their shared source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Every bulk group of this thread complete (writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit: thread t gets row (lane base + t), 32 columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major operand tile laid out in
// 128-byte-swizzled 8-row atoms (row pitch 128 B, atom stride 1024 B), as
// written by TMA with CU_TENSOR_MAP_SWIZZLE_128B and a 64-element bf16 box.
// Fields (tcgen05 smem descriptor): start>>4 [0,14), LBO>>4 [16,30) (unused
// for swizzled K-major; 1), SBO>>4 [32,46) = 1024>>4, version 1 at [46,48),
// base offset 0, layout SWIZZLE_128B = 2 at [61,64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
    d |= static_cast<uint64_t>(1) << 16;
    d |= static_cast<uint64_t>(1024 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Shared-memory descriptor for an MN-major operand in 128-byte-swizzled
// atoms: 64 16-bit elements of the MN dimension per 128-byte row, K rows at
// a 128-byte pitch, 8-row groups SBO = 1024 bytes apart.  Used for V in
// O = P V (V stored [key][dim], dims contiguous).  LBO (stride between
// 64-element MN groups) is set to lbo_bytes.
__device__ __forceinline__ uint64_t sw128_desc_mn(uint32_t smem_addr, uint32_t lbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= static_cast<uint64_t>(1024 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B of the
// same 16-bit type (format 0 = f16, 1 = bf16 at bits 7-9 and 10-12), both
// K-major, N>>3 at bits 17-22, M>>4 at bits 24-28.
__host__ __device__ constexpr uint32_t idesc_f32acc(int m, int n, bool bf16, bool b_mn_major = false) {
    return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// ---- 16-bit element helpers (bf16 / f16)
template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
    return v;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
    return __float2half_rn(v);
}
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t v);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t v) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162 *>(&v));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t v) {
    return __half22float2(*reinterpret_cast<__half2 *>(&v));
}

inline bool is_16bit(int dtype) { return dtype == P3D_BF16 || dtype == P3D_F16; }
inline size_t dtype_size(int dtype) { return dtype == P3D_F32 ? 4 : 2; }

// Dispatch a templated launch on a p3d_dtype (float / bf16 / f16).
#define P3D_DISPATCH(dtype, T, ...)                 \
    do {                                            \
        if ((dtype) == P3D_F32) {                   \
            using T = float;                        \
            __VA_ARGS__;                            \
        } else if ((dtype) == P3D_BF16) {           \
            using T = __nv_bfloat16;                \
            __VA_ARGS__;                            \
        } else {                                    \
            using T = __half;                       \
            __VA_ARGS__;                            \
        }                                           \
    } while (0)

// ---- misc math
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// GELU, tanh form: 0.5 x (1 + tanh(y)) with y = sqrt(2/pi) (x + 0.044715 x^3),
// with the hardware tanh approximation (tanh.approx.f32: one MUFU op,
// relative error about 2^-11, at the 16-bit output rounding of the MLP
// activations).
__device__ __forceinline__ float gelu_tanh_f(float x) {
    const float y = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(y));
    const float hx = 0.5f * x;
    return fmaf(hx, t, hx);
}
// SiLU x / (1 + exp(-x)) with the fast exp and divide (a few ulp; for
// x < -87 the denominator exceeds 2^126 and the result flushes to 0, as the
// exact value underflows there too).
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ int batch_of_row(const int32_t *offsets, int nbatch, int64_t row) {
    int b = 0;
    while (b + 1 < nbatch && row >= offsets[b + 1]) ++b;
    return b;
}

// Statistics of the CFG guidance rescale (sparse_batch_std,
// src/flow_sampler.cpp:164-198): per batch item b, stats[4b .. 4b+3] +=
// (sum, sum of squares) of x0(pos) and of x0(cfg), x0 = a x - (sigma_min +
// a t) v with a = 1 - sigma_min and the CFG prediction g v_pos + (1 - g)
// v_neg (v_pos when v_neg is null).  Each warp takes kStatsRowsPerWarp
// consecutive rows, its lanes stride over their elements, and it flushes its
// double partials with one set of atomics per batch segment (rows are
// contiguous by batch), instead of per row on the same four addresses.
constexpr int kStatsRowsPerWarp = 64;
__device__ __forceinline__ void cfg_stats_rows(const float *__restrict__ x, const float *__restrict__ vp,
                                               const float *__restrict__ vn, int64_t n, int C,
                                               const int32_t *__restrict__ offsets, int nbatch, float t, float g,
                                               float sigma_min, double *__restrict__ stats) {
    const int64_t warp_id = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t r0 = warp_id * kStatsRowsPerWarp;
    if (r0 >= n) return;
    const int64_t r1 = r0 + kStatsRowsPerWarp < n ? r0 + kStatsRowsPerWarp : n;
    const float a = 1.0f - sigma_min, bb = sigma_min + a * t;
    int b = batch_of_row(offsets, nbatch, r0);
    int64_t rs = r0;
    while (rs < r1) {
        const int64_t bend = offsets[b + 1];
        const int64_t re = bend < r1 ? bend : r1;
        if (re <= rs) {  // item b ends before rs (an empty item): move on; past the last item: stop
            if (b + 1 < nbatch) {
                ++b;
                continue;
            }
            break;
        }
        double s0 = 0, q0 = 0, s1 = 0, q1 = 0;
        for (int64_t e = rs * C + lane; e < re * C; e += 32) {
            const float p = vp[e];
            const float pred = vn ? g * p + (1.0f - g) * vn[e] : p;
            const float xp = a * x[e] - bb * p;
            const float xc = a * x[e] - bb * pred;
            s0 += xp;
            q0 += static_cast<double>(xp) * xp;
            s1 += xc;
            q1 += static_cast<double>(xc) * xc;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            s0 += __shfl_xor_sync(0xffffffffu, s0, o);
            q0 += __shfl_xor_sync(0xffffffffu, q0, o);
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            q1 += __shfl_xor_sync(0xffffffffu, q1, o);
        }
        if (lane == 0) {
            atomicAdd(stats + 4 * b + 0, s0);
            atomicAdd(stats + 4 * b + 1, q0);
            atomicAdd(stats + 4 * b + 2, s1);
            atomicAdd(stats + 4 * b + 3, q1);
        }
        rs = re;
    }
}

}  // namespace p3d
