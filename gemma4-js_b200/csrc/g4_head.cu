// g4_head.cu -- the tied bf16 LM head: logits = x . E^T in FP32.
//
// Replaces the BF16_HEAD shader (custom-webgpu/gpu-runtime.js:1265-1277), run by the
// reference as 64 dispatches of 4096 vocabulary rows each with one thread per row
// (gemma4-webgpu.js:170-188, :413-419).  The 805 MB bf16 embedding stays resident;
// M <= 16 rows use a bulk-copy + mma.m16n8k16 GEMV (HBM-bound), more rows use the
// tcgen05 GEMM with the bf16 operand loaded by TMA.  The softcap and the argmax are
// g4_softcap_argmax (g4_glue.cu).
#include "g4_common.cuh"
#include "g4_glue.cuh"
#include "g4_linear.cuh"
#include "g4_tcgen05.cuh"

#include "g4_dense.cuh"

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


// ---- fused head: logits tiles on tcgen05, softcap + greedy pick in the epilogue ------
// Tiles of 128 tokens (MMA M, TMEM lanes) x 256 vocabulary rows (MMA N): A = x and B =
// the bf16 table, both by TMA (128-byte swizzle) into a 4-stage ring; one thread issues
// 8 MMAs per pair of stages; the accumulator is double-buffered in TMEM (2 x 256 columns)
// so the epilogue of a tile overlaps the next tile's MMAs.  Epilogue warp w owns TMEM lane
// quarter w % 4 (32 tokens) and one half of the tile's columns: each thread reduces its
// token's 128 logits in registers (softcap, then the lowest index of the largest value)
// and writes one (value, index) pair; the logits never reach memory.
constexpr int HM = 128, HN = 256, HK = 64;
constexpr int kHStages = 4;
constexpr int kHEpi = 8;
constexpr int kHThreads = (2 + kHEpi) * 32;
constexpr int kHABytes = HM * HK * 2;              // 16 KB
constexpr int kHStageBytes = kHABytes + HN * HK * 2;  // + 32 KB
constexpr int kHSmem = kHStages * kHStageBytes + 256 + 1024;

struct HeadParams {
    int M, N, KB, MT, NT;  // KB = 64-column blocks of K; MT token tiles, NT vocabulary tiles
    float cap;
    float2* part;          // [M][2 * NT] (value, index bits)
    uint32_t* err;
};

__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

__global__ void __launch_bounds__(kHThreads, 1)
head_argmax_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                   const HeadParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kHStages * kHStageBytes);
    uint64_t* empty = full + kHStages;
    uint64_t* acc_full = empty + kHStages;  // [2]
    uint64_t* acc_empty = acc_full + 2;     // [2]
    uint32_t* tslot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = p.MT * p.NT;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kHStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kHEpi);
        }
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tslot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    pdl_trigger();
    if (warp >= 2) pdl_wait();

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tensor_map(&xmap);
            prefetch_tensor_map(&wmap);
            int pre = 0;  // the table is immutable: its first boxes before the predecessor wait
            for (int t = blockIdx.x; t < ntiles && pre < kHStages; t += gridDim.x)
                for (int kb = 0; kb < p.KB && pre < kHStages; ++kb, ++pre) {
                    mbar_arrive_expect_tx(&full[pre], kHStageBytes);
                    tma_load_2d(smem + pre * kHStageBytes + kHABytes, &wmap, &full[pre], kb * HK, (t / p.MT) * HN);
                }
            pdl_wait();
            bool ok = true;
            int g = 0;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const int mt = t % p.MT, nt = t / p.MT;
                for (int kb = 0; kb < p.KB; ++kb, ++g) {
                    const int s = g % kHStages;
                    if (g >= kHStages) {
                        if (!mbar_wait(&empty[s], ((g / kHStages) - 1) & 1, p.err, 0x201)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&full[s], kHStageBytes);
                        tma_load_2d(smem + s * kHStageBytes + kHABytes, &wmap, &full[s], kb * HK, nt * HN);
                    }
                    tma_load_2d(smem + s * kHStageBytes, &xmap, &full[s], kb * HK, mt * HM);
                }
            }
            for (int j = g > kHStages ? g - kHStages : 0; j < g; ++j)
                mbar_wait(&full[j % kHStages], (j / kHStages) & 1, p.err, 0x202);
        }
        __syncwarp();
    } else if (warp == 1) {
        // -------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = mma_idesc_bf16(HM, HN);
            bool ok = true;
            int g = 0, tj = 0;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tj) {
                const int ab = tj & 1;
                if (tj >= 2 && !mbar_wait(&acc_empty[ab], ((tj >> 1) - 1) & 1, p.err, 0x203)) break;
                tc_fence_after();
                const uint32_t acc = tmem + ab * HN;
                for (int kb = 0; kb < p.KB && ok; kb += 2) {
                    const int n = min(2, p.KB - kb);
                    for (int u = 0; u < n && ok; ++u)
                        ok = mbar_wait(&full[(g + u) % kHStages], ((g + u) / kHStages) & 1, p.err, 0x204);
                    if (!ok) break;
                    tc_fence_after();
                    for (int u = 0; u < n; ++u) {
                        const uint32_t a0 = smem_u32(smem + ((g + u) % kHStages) * kHStageBytes), b0 = a0 + kHABytes;
#pragma unroll
                        for (int ks = 0; ks < HK / 16; ++ks)
                            tc_mma_ss(acc, sw128_desc(a0 + ks * 32), sw128_desc(b0 + ks * 32), idesc,
                                      (kb + u > 0 || ks > 0) ? 1u : 0u);
                    }
                    for (int u = 0; u < n; ++u) tc_commit(&empty[(g + u) % kHStages]);
                    g += n;
                }
                tc_commit(&acc_full[ab]);  // tile complete (or abandoned after a timeout)
            }
        }
        __syncwarp();
    } else {
        // ----------------------------------------------------- softcap + argmax
        const int q = warp & 3, e = (warp - 2) >> 2;
        int tj = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tj) {
            const int ab = tj & 1, mt = t % p.MT, nt = t / p.MT;
            if (!mbar_wait_warp(&acc_full[ab], (tj >> 1) & 1, p.err, 0x205)) break;
            tc_fence_after();
            const uint32_t tq = tmem + ab * HN + ((uint32_t)(32 * q) << 16) + 128 * e;
            const int n0 = nt * HN + 128 * e;
            // A thread meets its columns in increasing index order and the softcap is
            // non-decreasing, so a logit no larger than the largest raw logit seen so far
            // can neither exceed the pick nor win a tie against it (its index is higher):
            // the softcap is evaluated only on a new raw maximum.
            float bv = -INFINITY, rmax = -INFINITY;
            int bi = 0x7fffffff;
            for (int c = 0; c < 128; c += 32) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tq + c, v);
                tmem_ld_wait(v);
                if (c == 96) {  // the accumulator buffer is free for the tile after next
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[ab]);
                }
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    const int n = n0 + c + jj;
                    const float raw = __uint_as_float(v[jj]);
                    // NaN skipped, as g4_softcap_argmax; the first valid column always taken
                    if (n < p.N && raw == raw && (raw > rmax || bi == 0x7fffffff)) {
                        rmax = raw;
                        const float val = p.cap > 0.f ? tanhf(raw / p.cap) * p.cap : raw;
                        if (val > bv || bi == 0x7fffffff) {
                            bv = val;
                            bi = n;
                        }
                    }
                }
            }
            const int m = mt * HM + 32 * q + lane;
            if (m < p.M) p.part[(size_t)m * (2 * p.NT) + nt * 2 + e] = make_float2(bv, __int_as_float(bi));
        }
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
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

g4_status g4_dense_argmax(g4_ctx* ctx, const g4_dense* d, const void* x_bf16, int M, float cap, int32_t* ids_out,
                          float* vals_out) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!d || !x_bf16 || !ids_out || M < 0) return g4::set_error(G4_ERR_INVALID, "g4_dense_argmax: bad arguments");
    if (M == 0) return G4_OK;
    if (reinterpret_cast<uintptr_t>(x_bf16) % 16 != 0 || d->K % 8 != 0)
        return g4::set_error(G4_ERR_INVALID, "g4_dense_argmax: x must be 16-byte aligned and K a multiple of 8");
    static std::atomic<uint64_t> attr_set{0};
    if (!(attr_set.load() & (1ull << ctx->device))) {
        G4_CHECK_CUDA(cudaFuncSetAttribute(head_argmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kHSmem));
        attr_set.fetch_or(1ull << ctx->device);
    }
    HeadParams p{};
    p.M = M;
    p.N = d->N;
    p.KB = (d->K + HK - 1) / HK;
    p.MT = (M + HM - 1) / HM;
    p.NT = (d->N + HN - 1) / HN;
    p.cap = cap;
    p.err = ctx->d_err;
    const int nparts = 2 * p.NT;
    st = g4::ensure_workspace(ctx, (size_t)M * nparts * sizeof(float2));
    if (st) return st;
    p.part = static_cast<float2*>(ctx->ws);
    CUtensorMap xmap;
    st = g4::encode_tensor_map_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, const_cast<void*>(x_bf16), d->K, M,
                                  (uint64_t)d->K * 2, HK, HM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    const long long ntiles = (long long)p.MT * p.NT;
    const unsigned grid = (unsigned)std::min<long long>(ntiles, ctx->num_sms);
    st = g4::launch(ctx, "head_argmax_kernel", head_argmax_kernel, dim3(grid), dim3(kHThreads), kHSmem, 1, xmap,
                    d->bmap, p);
    if (st) return st;
    return g4::launch_argmax_final(ctx, p.part, nparts, M, ids_out, vals_out);
}

}  // extern "C"
