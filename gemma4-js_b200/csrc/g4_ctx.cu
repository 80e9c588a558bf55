// g4_ctx.cu -- context, errors, workspace and tensor-map plumbing of libg4w4.so.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "g4_common.cuh"

namespace {
thread_local std::string t_last_error;
std::atomic<uint64_t> g_launches{0};
}  // namespace

namespace g4 {

g4_status set_error(g4_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return st;
}

g4_status cuda_error(cudaError_t e, const char* what) {
    return set_error(e == cudaErrorMemoryAllocation ? G4_ERR_OOM : G4_ERR_CUDA, "%s: %s (%s)",
                     what, cudaGetErrorString(e), cudaGetErrorName(e));
}

void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

g4_status use_device(const g4_ctx* ctx) {
    if (!ctx) return set_error(G4_ERR_INVALID, "null context");
    int cur = -1;
    G4_CHECK_CUDA(cudaGetDevice(&cur));
    if (cur != ctx->device) G4_CHECK_CUDA(cudaSetDevice(ctx->device));
    return G4_OK;
}

g4_status ensure_workspace(g4_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->ws_bytes) return G4_OK;
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    want = (want + 4095) & ~size_t(4095);
    void* fresh = nullptr;
    G4_CHECK_CUDA(cudaMalloc(&fresh, want));
    if (ctx->ws) ctx->ws_retired.push_back(ctx->ws);  // queued kernels or captured graphs may still use it
    ctx->ws = fresh;
    ctx->ws_bytes = want;
    return G4_OK;
}

g4_status ensure_stage(g4_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->stage_bytes) return G4_OK;
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    want = (want + 4095) & ~size_t(4095);
    void* fresh = nullptr;
    G4_CHECK_CUDA(cudaMalloc(&fresh, want));
    if (ctx->stage) ctx->stage_retired.push_back(ctx->stage);
    ctx->stage = fresh;
    ctx->stage_bytes = want;
    return G4_OK;
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

g4_status encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, void* base,
                               uint64_t inner, uint64_t outer, uint64_t row_pitch_bytes,
                               uint32_t box_inner, uint32_t box_outer,
                               CUtensorMapSwizzle swizzle) {
    auto fn = get_encode_fn();
    if (!fn) return set_error(G4_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_pitch_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dtype, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(G4_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu box %u x %u",
                         (int)r, (unsigned long long)inner, (unsigned long long)outer, box_inner,
                         box_outer);
    return G4_OK;
}

}  // namespace g4

extern "C" {

g4_status g4_ctx_create(int device, void* stream, g4_ctx** out) {
    if (!out) return g4::set_error(G4_ERR_INVALID, "g4_ctx_create: null out");
    *out = nullptr;
    int n = 0;
    G4_CHECK_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n)
        return g4::set_error(G4_ERR_INVALID, "g4_ctx_create: device %d of %d", device, n);
    G4_CHECK_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    G4_CHECK_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10 || prop.minor != 0)
        return g4::set_error(G4_ERR_UNSUPPORTED,
                             "g4_ctx_create: device %d is sm_%d%d; libg4w4 is built for sm_100a",
                             device, prop.major, prop.minor);
    g4_ctx* c = new g4_ctx();
    c->device = device;
    c->stream = static_cast<cudaStream_t>(stream);
    c->num_sms = prop.multiProcessorCount;
    cudaError_t e = cudaMalloc(&c->d_err, 2 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(c->d_err, 0, 2 * sizeof(uint32_t));
    if (e != cudaSuccess) {
        delete c;
        return g4::cuda_error(e, "g4_ctx_create");
    }
    *out = c;
    return G4_OK;
}

g4_status g4_ctx_destroy(g4_ctx* ctx) {
    if (!ctx) return G4_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->d_err);
    cudaFree(ctx->ws);
    for (void* p : ctx->ws_retired) cudaFree(p);
    cudaFree(ctx->stage);
    for (void* p : ctx->stage_retired) cudaFree(p);
    cudaFree(ctx->d_ids);
    delete ctx;
    return G4_OK;
}

g4_status g4_ctx_set_stream(g4_ctx* ctx, void* stream) {
    if (!ctx) return g4::set_error(G4_ERR_INVALID, "null context");
    ctx->stream = static_cast<cudaStream_t>(stream);
    return G4_OK;
}

g4_status g4_ctx_set_pdl(g4_ctx* ctx, int enable) {
    if (!ctx) return g4::set_error(G4_ERR_INVALID, "null context");
    ctx->pdl = enable != 0;
    return G4_OK;
}

g4_status g4_stream_sync(g4_ctx* ctx) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    G4_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
    return G4_OK;
}

g4_status g4_ctx_check_device(g4_ctx* ctx, uint32_t* flags) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    uint32_t hw[2] = {0, 0};
    G4_CHECK_CUDA(cudaMemcpyAsync(hw, ctx->d_err, sizeof(hw), cudaMemcpyDeviceToHost, ctx->stream));
    G4_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
    const uint32_t h = hw[0];
    if (flags) *flags = h;
    if (h) {
        G4_CHECK_CUDA(cudaMemsetAsync(ctx->d_err, 0, sizeof(hw), ctx->stream));
        G4_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
        if (h & G4_DEVERR_TIMEOUT)
            return g4::set_error(G4_ERR_TIMEOUT, "a device-side bounded wait timed out (flags 0x%x, wait site %u)", h,
                                 hw[1]);
        return g4::set_error(G4_ERR_DEVICE, "a kernel saw an out-of-range index (flags 0x%x)", h);
    }
    return G4_OK;
}

}  // extern "C"

namespace {
// One thread waits on an mbarrier that nothing arrives on, through the bounded wait every
// kernel of the library uses (mbar_wait): it gives up after kWaitLimitNs, raises
// G4_DEVERR_TIMEOUT with `site` and returns.
__global__ void wait_timeout_selftest_kernel(uint32_t* err, uint32_t site) {
    using namespace g4dev;
    __shared__ __align__(8) uint64_t bar;
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_wait(&bar, 0, err, site);
}
}  // namespace

extern "C" {

g4_status g4_selftest_wait_timeout(g4_ctx* ctx, uint32_t site) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    wait_timeout_selftest_kernel<<<1, 1, 0, ctx->stream>>>(ctx->d_err, site);
    G4_CHECK_CUDA(cudaGetLastError());
    return G4_OK;
}

const char* g4_last_error_string(void) { return t_last_error.c_str(); }

const char* g4_version(void) { return "g4w4 0.1 sm_100a"; }

uint64_t g4_kernel_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
