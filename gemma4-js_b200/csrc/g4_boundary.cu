// g4_boundary.cu -- the reference's f32 buffer convention at the C ABI.
//
// GPUOps.w4 and GPUOps.attention (custom-webgpu/gpu-runtime.js:1316-1324, :1357-1365) take
// f32 GPU buffers and return new f32 buffers (`emptyF32`); the reference's model graph keeps
// every activation in f32 (gemma4-webgpu.js:215-310).  The W4A16 kernels of this library
// compute on bf16 activations with FP32 accumulation, so these entry points round the f32
// inputs to bf16 (round to nearest even, the reference's roundFloat32ToBF16 rule,
// official-w4a16.js:34-48) into a context staging buffer, run the bf16 kernels, and hand
// back f32 (the linear writes f32 directly; the attention's bf16 rows are widened exactly).
#include "g4_common.cuh"

namespace {

using namespace g4dev;

// dst[i] = src[i] for n elements: f32 -> bf16 rounds to nearest even (bit-identical to
// roundFloat32ToBF16), bf16 -> f32 is exact, equal dtypes copy the bits (a bf16 -> f32 ->
// bf16 round trip is the identity, NaN payloads included).
__global__ void __launch_bounds__(256) convert_kernel(const void* __restrict__ src, int src_f32,
                                                      void* __restrict__ dst, int dst_f32, long long n) {
    pdl_trigger();
    pdl_wait();
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float v = src_f32 ? static_cast<const float*>(src)[i]
                                : bf16_bits_to_f32(static_cast<const uint16_t*>(src)[i]);
        if (dst_f32)
            static_cast<float*>(dst)[i] = v;
        else
            static_cast<uint16_t*>(dst)[i] = (uint16_t)f32_to_bf16_bits(v);
    }
}

g4_status convert(g4_ctx* ctx, const void* src, int src_f32, void* dst, int dst_f32, long long n) {
    if (n <= 0) return G4_OK;
    const long long blocks = (n + 255) / 256;
    const unsigned grid = (unsigned)(blocks < 8LL * ctx->num_sms ? blocks : 8LL * ctx->num_sms);
    return g4::launch(ctx, "convert_kernel", convert_kernel, dim3(grid), dim3(256), 0, 1, src, src_f32, dst, dst_f32, n);
}

size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

}  // namespace

extern "C" {

g4_status g4_convert(g4_ctx* ctx, const void* src, g4_dtype src_dtype, void* dst, g4_dtype dst_dtype, long long n) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (n < 0) return g4::set_error(G4_ERR_INVALID, "g4_convert: n = %lld", n);
    if (n == 0) return G4_OK;
    if (!src || !dst) return g4::set_error(G4_ERR_INVALID, "g4_convert: null argument");
    if ((src_dtype != G4_F32 && src_dtype != G4_BF16) || (dst_dtype != G4_F32 && dst_dtype != G4_BF16))
        return g4::set_error(G4_ERR_INVALID, "g4_convert: dtypes %d -> %d", (int)src_dtype, (int)dst_dtype);
    return convert(ctx, src, src_dtype == G4_F32, dst, dst_dtype == G4_F32, n);
}

g4_status g4_linear_w4a16_f32(g4_ctx* ctx, const g4_linear* lin, const float* x, int M, float* y) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!lin || !x || !y) return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16_f32: null argument");
    if (M < 0) return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16_f32: M = %d", M);
    if (M == 0) return G4_OK;
    int K = 0, N = 0;
    st = g4_linear_shape(lin, &K, &N);
    if (st) return st;
    const long long n = (long long)M * K;
    st = g4::ensure_stage(ctx, align256((size_t)n * 2));
    if (st) return st;
    st = convert(ctx, x, 1, ctx->stage, 0, n);
    if (st) return st;
    return g4_linear_w4a16(ctx, lin, ctx->stage, M, y, G4_F32);
}

g4_status g4_attention_f32(g4_ctx* ctx, const float* q, const g4_kv* kv, int rows, int heads, int hd, int keylen,
                           int qpos0, int sliding, int window, float* out) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!kv || !q || !out) return g4::set_error(G4_ERR_INVALID, "g4_attention_f32: null argument");
    if (rows < 0 || heads < 1 || hd < 1)
        return g4::set_error(G4_ERR_INVALID, "g4_attention_f32: rows %d heads %d hd %d", rows, heads, hd);
    if (rows == 0) return G4_OK;
    const long long n = (long long)rows * heads * hd;
    const size_t half = align256((size_t)n * 2);
    st = g4::ensure_stage(ctx, 2 * half);
    if (st) return st;
    uint8_t* qs = static_cast<uint8_t*>(ctx->stage);
    uint8_t* os = qs + half;
    st = convert(ctx, q, 1, qs, 0, n);
    if (st) return st;
    st = g4_attention(ctx, qs, kv, rows, heads, hd, keylen, qpos0, sliding, window, os);
    if (st) return st;
    return convert(ctx, os, 0, out, 1, n);
}

}  // extern "C"
