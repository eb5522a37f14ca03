// Neighbour map whose hash-table scratch is a file-scope device array, so the
// call allocates no device memory: p3d_neighbor_map27_static.
//
// The table (keys then values, the layout p3d_neighbor_map27_ws carves out
// of caller scratch) lives in g_nbr_table, which every GPU that loads the
// library holds until the process exits.  Host code cannot use the symbol
// itself as a device address, so every call asks the runtime for the
// array's address on ctx's device (cudaGetSymbolAddress, with that device
// current).  Nothing is cached: after a device reset the next call gets the
// address in the new context.  The first call on a device also loads the
// module there, which is why that call must come before any stream capture.
#include "p3d_common.cuh"

namespace {

// Largest table: 2^20 slots (8 MiB of keys + 4 MiB of values).  The table is
// sized like p3d_coord_hash_capacity (a power of two >= 2n, at least 64), so
// it serves up to P3D_NBR_STATIC_MAX_POINTS = 2^19 points.
constexpr int64_t kSlots = int64_t(1) << 20;
constexpr int64_t kMaxPoints = kSlots / 2;
static_assert(kMaxPoints == P3D_NBR_STATIC_MAX_POINTS, "static table size and header limit disagree");

// [kSlots] uint64 keys, then [kSlots] int32 values (kSlots/2 uint64 words).
static __device__ __align__(256) uint64_t g_nbr_table[kSlots + kSlots / 2];

// Device address of g_nbr_table on ctx->device.
int table_address(p3d_ctx *ctx, void **out) {
    int prev = -1;
    P3D_CUDA(ctx, cudaGetDevice(&prev));
    if (prev != ctx->device) P3D_CUDA(ctx, cudaSetDevice(ctx->device));
    void *ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_nbr_table);
    if (prev != ctx->device) cudaSetDevice(prev);
    if (e != cudaSuccess)
        return p3d::set_error(ctx, P3D_ERR_CUDA,
                              std::string("p3d_neighbor_map27_static: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    *out = ptr;
    return P3D_OK;
}

}  // namespace

extern "C" int p3d_neighbor_map27_static(p3d_ctx *ctx, const int32_t *coords, int64_t n, int32_t *nbr_out) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, coords && nbr_out, "p3d_neighbor_map27_static: null pointer");
    P3D_REQUIRE(ctx, n >= 0, "p3d_neighbor_map27_static: negative point count");
    if (n > kMaxPoints)
        return p3d::set_error(ctx, P3D_ERR_INVALID,
                              "p3d_neighbor_map27_static: " + std::to_string(n) +
                                  " points exceed the static table's maximum of " + std::to_string(kMaxPoints) +
                                  " (use p3d_neighbor_map27_ws with caller scratch)");
    void *table = nullptr;
    int rc = table_address(ctx, &table);
    if (rc) return rc;
    // Only the first `cap` slots are used; p3d_coord_hash_build resets their
    // keys to empty before inserting, which clears the previous call's keys.
    const int64_t cap = p3d_coord_hash_capacity(n);
    uint64_t *keys = static_cast<uint64_t *>(table);
    int32_t *vals = reinterpret_cast<int32_t *>(keys + kSlots);
    rc = p3d_coord_hash_build(ctx, coords, n, keys, vals, cap);
    if (rc) return rc;
    return p3d_neighbor_map27(ctx, coords, n, keys, vals, cap, nbr_out);
}
