// g4_head.cu -- the tied bf16 LM head: logits = x . E^T in FP32.
//
// Replaces the BF16_HEAD shader (custom-webgpu/gpu-runtime.js:1265-1277), run by the
// reference as 64 dispatches of 4096 vocabulary rows each with one thread per row
// (gemma4-webgpu.js:170-188, :413-419).  The 805 MB bf16 embedding stays resident;
// M <= 16 rows use a bulk-copy + mma.m16n8k16 GEMV (HBM-bound), more rows use the
// tcgen05 GEMM with the bf16 operand loaded by TMA.  The softcap and the argmax are
// g4_softcap_argmax (g4_glue.cu).
#include "g4_common.cuh"
#include "g4_linear.cuh"

struct g4_dense {
    g4_ctx* ctx = nullptr;
    int K = 0, N = 0;
    uint16_t* w = nullptr;  // [N, K] bf16
    CUtensorMap bmap;       // boxes of 64 columns x 256 rows, 128B swizzle (tcgen05 B operand)
};

namespace {

using namespace g4dev;

constexpr int kHeadWarps = 4;

// 16 rows of W per CTA; W rows and the M activation rows are staged in shared memory
// by bulk copies (row pitch padded by 16 B so ldmatrix is conflict-free); each warp
// covers a quarter of K; the quarters are summed in shared memory.
template <int kNB>
__global__ void __launch_bounds__(kHeadWarps * 32) head_gemv_kernel(const uint16_t* __restrict__ w, int N, int K,
                                                                    const uint16_t* __restrict__ x, int M,
                                                                    float* __restrict__ y, uint32_t* err) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int pitch = K * 2 + 16;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
    uint8_t* wsm = sm + 128;
    uint8_t* xsm = wsm + 16 * pitch;
    float* red = reinterpret_cast<float*>(xsm + kNB * 8 * pitch);  // [warps][kNB*4][32]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int n0 = blockIdx.x * 16;
    const int rows = min(16, N - n0);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(bar, (uint32_t)(rows + M) * K * 2);
        for (int r = 0; r < rows; ++r) bulk_load(wsm + r * pitch, w + (size_t)(n0 + r) * K, K * 2, bar);
    }
    pdl_wait();  // the head rows are immutable; x comes from the predecessor
    if (threadIdx.x == 0)
        for (int b = 0; b < M; ++b) bulk_load(xsm + b * pitch, x + (size_t)b * K, K * 2, bar);
    // rows past N read as zero
    for (int i = threadIdx.x; i < (16 - rows) * (K / 8); i += blockDim.x) {
        const int r = rows + i / (K / 8), c = i % (K / 8);
        *reinterpret_cast<uint4*>(wsm + r * pitch + c * 16) = make_uint4(0, 0, 0, 0);
    }
    const bool ok = mbar_wait(bar, 0, err);
    __syncthreads();
    float acc[kNB][4];
#pragma unroll
    for (int j = 0; j < kNB; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    if (ok) {
        const int steps = K / 16, per = (steps + kHeadWarps - 1) / kHeadWarps;
        const int s0 = warp * per, s1 = min(steps, s0 + per);
        const int mj = lane >> 3, mr = lane & 7;
        const uint32_t wbase = smem_u32(wsm) + (uint32_t)(((mj & 1) * 8 + mr) * pitch + (mj >> 1) * 16);
        for (int s = s0; s < s1; ++s) {
            uint32_t a[4];
            ldmatrix_x4(a, wbase + s * 32);
#pragma unroll
            for (int j = 0; j < kNB; ++j) {
                const int b = j * 8 + g;
                uint32_t bb[2] = {0u, 0u};
                if (b < M) {
                    const uint8_t* xr = xsm + b * pitch + s * 32 + t * 4;
                    bb[0] = *reinterpret_cast<const uint32_t*>(xr);
                    bb[1] = *reinterpret_cast<const uint32_t*>(xr + 16);
                }
                mma_bf16_16816(acc[j], a, bb, acc[j]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kNB; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[(warp * kNB * 4 + j * 4 + e) * 32 + lane] = acc[j][e];
    __syncthreads();
    if (warp != 0) return;
#pragma unroll
    for (int j = 0; j < kNB; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float v = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < kHeadWarps; ++w2) v += red[(w2 * kNB * 4 + j * 4 + e) * 32 + lane];
            const int n = n0 + g + ((e & 2) ? 8 : 0), b = j * 8 + 2 * t + (e & 1);
            if (n < N && b < M) y[(size_t)b * N + n] = v;
        }
}

}  // namespace

extern "C" {

g4_status g4_dense_create(g4_ctx* ctx, const void* w_bf16, int K, int N, int src_on_device, g4_dense** out) {
    if (!out) return g4::set_error(G4_ERR_INVALID, "g4_dense_create: null out");
    *out = nullptr;
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (K <= 0 || N <= 0 || K % 16 != 0 || N % 8 != 0)
        return g4::set_error(G4_ERR_UNSUPPORTED, "g4_dense_create: K=%d (multiple of 16) N=%d (multiple of 8)", K, N);
    g4_dense* d = new g4_dense();
    d->ctx = ctx;
    d->K = K;
    d->N = N;
    const size_t bytes = (size_t)N * K * 2;
    cudaError_t e = cudaMalloc(&d->w, bytes);
    if (e == cudaSuccess && w_bf16)
        e = cudaMemcpyAsync(d->w, w_bf16, bytes, src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                            ctx->stream);
    if (e == cudaSuccess && w_bf16 && !src_on_device) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        g4_dense_destroy(d);
        return g4::cuda_error(e, "g4_dense_create");
    }
    st = g4::encode_tensor_map_2d(&d->bmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d->w, K, N, (uint64_t)K * 2, 64, 256,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) {
        g4_dense_destroy(d);
        return st;
    }
    *out = d;
    return G4_OK;
}

g4_status g4_dense_destroy(g4_dense* d) {
    if (!d) return G4_OK;
    if (d->ctx) cudaSetDevice(d->ctx->device);
    cudaFree(d->w);
    delete d;
    return G4_OK;
}

g4_status g4_dense_weights(const g4_dense* d, void** w) {
    if (!d || !w) return g4::set_error(G4_ERR_INVALID, "g4_dense_weights: null argument");
    *w = d->w;
    return G4_OK;
}

g4_status g4_dense_matmul(g4_ctx* ctx, const g4_dense* d, const void* x_bf16, int M, float* y) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!d || !x_bf16 || !y || M < 0) return g4::set_error(G4_ERR_INVALID, "g4_dense_matmul: bad arguments");
    if (M == 0) return G4_OK;
    if (reinterpret_cast<uintptr_t>(x_bf16) % 16 != 0)
        return g4::set_error(G4_ERR_INVALID, "g4_dense_matmul: x must be 16-byte aligned");
    const uint16_t* x = static_cast<const uint16_t*>(x_bf16);
    if (M > 16) return g4::launch_gemm_bf16(ctx, d->bmap, d->N, d->K, x, M, y);
    const int nb = M <= 8 ? 1 : 2;
    const size_t smem = 128 + (size_t)(16 + nb * 8) * (d->K * 2 + 16) + kHeadWarps * nb * 4 * 32 * 4;
    if (smem > 220 * 1024) return g4::set_error(G4_ERR_UNSUPPORTED, "g4_dense_matmul: K=%d too large for the GEMV", d->K);
    static std::atomic<uint64_t> attr_set{0};
    if (!(attr_set.load() & (1ull << ctx->device))) {
        G4_CHECK_CUDA(cudaFuncSetAttribute(head_gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        G4_CHECK_CUDA(cudaFuncSetAttribute(head_gemv_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        attr_set.fetch_or(1ull << ctx->device);
    }
    const unsigned grid = (unsigned)((d->N + 15) / 16);
    const uint16_t* w = d->w;
    if (nb == 1)
        return g4::launch(ctx, "head_gemv_kernel", head_gemv_kernel<1>, dim3(grid), dim3(kHeadWarps * 32), smem, 1, w,
                          d->N, d->K, x, M, y, ctx->d_err);
    return g4::launch(ctx, "head_gemv_kernel", head_gemv_kernel<2>, dim3(grid), dim3(kHeadWarps * 32), smem, 1, w, d->N,
                      d->K, x, M, y, ctx->d_err);
}

}  // extern "C"
