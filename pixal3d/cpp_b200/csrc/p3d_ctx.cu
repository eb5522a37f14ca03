// Context, error reporting and precision conversions.
#include <cstdio>

#include "p3d_common.cuh"

namespace p3d {

int set_error(p3d_ctx *ctx, int status, const std::string &msg) {
    if (ctx) ctx->error = msg;
    return status;
}

int check_launch(p3d_ctx *ctx, const char *what) {
    ++ctx->launches;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ctx, P3D_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    return P3D_OK;
}

namespace {

template <typename TI, typename TO>
__global__ void convert_kernel(const TI *__restrict__ x, int64_t n, TO *__restrict__ y) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) y[i] = from_f32<TO>(to_f32(x[i]));
}

}  // namespace
}  // namespace p3d

using namespace p3d;

extern "C" int p3d_version(void) { return 1; }

extern "C" int p3d_ctx_create(int device, void *stream, p3d_ctx **out) {
    if (!out) return P3D_ERR_INVALID;
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= device || device < 0) return P3D_ERR_NO_DEVICE;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return P3D_ERR_NO_DEVICE;
    if (prop.major != 10) return P3D_ERR_NO_DEVICE;  // built for sm_100a only
    // The fault flag lives on `device`; the caller's current device is restored.
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) return P3D_ERR_CUDA;
    if (prev != device && cudaSetDevice(device) != cudaSuccess) return P3D_ERR_CUDA;
    p3d_ctx *ctx = new p3d_ctx();
    ctx->device = device;
    ctx->stream = static_cast<cudaStream_t>(stream);
    ctx->num_sms = prop.multiProcessorCount;
    const bool ok =
        cudaMalloc(&ctx->fault, sizeof(int)) == cudaSuccess && cudaMemset(ctx->fault, 0, sizeof(int)) == cudaSuccess;
    if (prev != device) cudaSetDevice(prev);
    if (!ok) {
        if (ctx->fault) cudaFree(ctx->fault);
        delete ctx;
        return P3D_ERR_CUDA;
    }
    *out = ctx;
    return P3D_OK;
}

extern "C" int p3d_ctx_destroy(p3d_ctx *ctx) {
    if (!ctx) return P3D_OK;
    if (ctx->fault) cudaFree(ctx->fault);
    delete ctx;
    return P3D_OK;
}

extern "C" int p3d_ctx_set_stream(p3d_ctx *ctx, void *stream) {
    if (!ctx) return P3D_ERR_INVALID;
    ctx->stream = static_cast<cudaStream_t>(stream);
    return P3D_OK;
}

extern "C" void *p3d_ctx_stream(const p3d_ctx *ctx) { return ctx ? ctx->stream : nullptr; }

extern "C" const char *p3d_last_error(const p3d_ctx *ctx) { return ctx ? ctx->error.c_str() : "null context"; }

extern "C" int64_t p3d_ctx_launch_count(const p3d_ctx *ctx) { return ctx ? ctx->launches : 0; }

extern "C" int p3d_ctx_check(p3d_ctx *ctx) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    int fault = 0;
    P3D_CUDA(ctx, cudaMemcpy(&fault, ctx->fault, sizeof(int), cudaMemcpyDeviceToHost));
    if (fault) {
        P3D_CUDA(ctx, cudaMemset(ctx->fault, 0, sizeof(int)));
        const char *what = fault == P3D_ERR_TIMEOUT     ? "device wait timed out"
                           : fault == P3D_ERR_HASH_FULL ? "coordinate hash table full"
                           : fault == P3D_ERR_DUPLICATE ? "sparse coordinates contain a duplicate point"
                           : fault == P3D_ERR_NONFINITE ? "non-finite value"
                                                        : "device fault";
        return set_error(ctx, fault, what);
    }
    return P3D_OK;
}

namespace p3d {
namespace {
// One thread waits, through the pipelines' bounded-wait routine, on phase 0 of
// an mbarrier of arrival count 1.  With `complete`, a thread of another warp
// makes that arrival (the wait succeeds); without it nothing does, so the wait
// runs out after limit_ns, latches P3D_ERR_TIMEOUT and the kernel returns.
// out[0] = 1 when the wait succeeded, out[1] = its duration in ns.
__global__ void wait_selftest_kernel(int complete, uint64_t limit_ns, int *fault, int64_t *out) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 32 && complete) mbar_arrive(&bar);
    if (threadIdx.x == 0) {
        const uint64_t t0 = globaltimer();
        const bool ok = mbar_wait_for(&bar, 0, fault, limit_ns);
        out[0] = ok ? 1 : 0;
        out[1] = static_cast<int64_t>(globaltimer() - t0);
    }
}
}  // namespace
}  // namespace p3d

extern "C" int p3d_wait_selftest(p3d_ctx *ctx, int complete, int64_t limit_ns, int64_t *out_host) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, out_host && limit_ns > 0 && limit_ns <= 5000000000ll,
                "p3d_wait_selftest: limit must be in (0, 5 s] and out non-null");
    DeviceGuard dg(ctx->device);
    int64_t *d = nullptr;
    P3D_CUDA(ctx, cudaMalloc(&d, 2 * sizeof(int64_t)));
    wait_selftest_kernel<<<1, 64, 0, ctx->stream>>>(complete, static_cast<uint64_t>(limit_ns), ctx->fault, d);
    int rc = check_launch(ctx, "wait_selftest");
    if (rc == P3D_OK) {
        cudaError_t e = cudaMemcpyAsync(out_host, d, 2 * sizeof(int64_t), cudaMemcpyDeviceToHost, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        rc = e == cudaSuccess ? p3d_ctx_check(ctx) : set_error(ctx, P3D_ERR_CUDA, cudaGetErrorString(e));
    }
    cudaFree(d);
    return rc;
}

extern "C" int p3d_convert(p3d_ctx *ctx, const void *x, int x_dtype, int64_t count, void *out, int out_dtype) {
    if (!ctx) return P3D_ERR_INVALID;
    P3D_REQUIRE(ctx, x && out, "p3d_convert: null pointer");
    P3D_REQUIRE(ctx, x_dtype >= P3D_F32 && x_dtype <= P3D_F16 && out_dtype >= P3D_F32 && out_dtype <= P3D_F16,
                "p3d_convert: bad dtype");
    if (count == 0) return P3D_OK;
    const unsigned grid = static_cast<unsigned>(ceil_div(count, 256));
    P3D_DISPATCH(x_dtype, TI, P3D_DISPATCH(out_dtype, TO, convert_kernel<TI, TO><<<grid, 256, 0, ctx->stream>>>(
                                                              static_cast<const TI *>(x), count, static_cast<TO *>(out))));
    return check_launch(ctx, "convert");
}

extern "C" int p3d_device_alloc(p3d_ctx *ctx, size_t bytes, void **out) {
    if (!ctx || !out) return P3D_ERR_INVALID;
    *out = nullptr;
    if (bytes == 0) bytes = 1;
    DeviceGuard dg(ctx->device);
    P3D_CUDA(ctx, cudaMalloc(out, bytes));
    return P3D_OK;
}

extern "C" int p3d_device_free(p3d_ctx *ctx, void *ptr) {
    if (!ctx) return P3D_ERR_INVALID;
    if (!ptr) return P3D_OK;
    DeviceGuard dg(ctx->device);
    P3D_CUDA(ctx, cudaFree(ptr));
    return P3D_OK;
}

extern "C" int p3d_copy_to_device(p3d_ctx *ctx, void *dst, const void *src, size_t bytes) {
    if (!ctx) return P3D_ERR_INVALID;
    if (bytes == 0) return P3D_OK;
    P3D_REQUIRE(ctx, dst && src, "p3d_copy_to_device: null pointer");
    DeviceGuard dg(ctx->device);
    P3D_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    return P3D_OK;
}

extern "C" int p3d_copy_to_host(p3d_ctx *ctx, void *dst, const void *src, size_t bytes) {
    if (!ctx) return P3D_ERR_INVALID;
    if (bytes == 0) return P3D_OK;
    P3D_REQUIRE(ctx, dst && src, "p3d_copy_to_host: null pointer");
    DeviceGuard dg(ctx->device);
    P3D_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    P3D_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    return P3D_OK;
}

extern "C" int p3d_ctx_synchronize(p3d_ctx *ctx) {
    if (!ctx) return P3D_ERR_INVALID;
    DeviceGuard dg(ctx->device);
    P3D_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    return p3d_ctx_check(ctx);
}
