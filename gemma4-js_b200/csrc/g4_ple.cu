// g4_ple.cu -- PLE W4 table on the device and the gather-dequant kernel.
//
// Replaces the reference's per-token shard byte gather on the CPU plus the WGSL
// dequant (custom-webgpu/gpu-runtime.js:218-256, :265-335, :487-527): here the whole
// [vocab, 8960] W4 table (1.32 GB) stays resident in HBM and one kernel gathers and
// dequantises the rows of a token batch straight into [T, 35, 256].
#include <stdio.h>

#include "g4_common.cuh"
#include "g4_ple.cuh"

namespace {

using namespace g4dev;

// One CTA per token, one thread per packed 32-bit word (8 columns) at a time.  Consecutive
// threads own consecutive words, so a warp loads 128 contiguous bytes of nibbles and stores
// 512 contiguous bytes of bf16 output in one instruction each.  The row's scales (560 bytes)
// go to shared memory first, one 16-byte load per 8 groups, issued together with the word
// loads: half the load instructions of a per-word scale load.  Each thread issues the loads
// of all its words, then decodes and stores them (8960 columns = 1120 words = 160 threads
// x 7).  The table's own width is compiled in (kWPR = 1120): without the per-word bounds
// checks and runtime strides the kernel measured 16.8 instead of 17.6 us per 4096 tokens;
// other widths take the generic instance (kWPR = 0).
//
// Decode (ple-w4-shard-reader.js:89-95): column c is nibble (c & 1) of byte c >> 1,
// i.e. bits 4c..4c+3 of the little-endian 32-bit word c >> 3; value = two's
// complement nibble * f32(scale), exact in f32.
constexpr int kPleThreads = 160;
constexpr int kPleWords = 7;
constexpr int kPleWidthWords = 1120;  // 8960 columns

// Word j of an output row: 8 columns from packed word w with the bf16 scale bits sb.
template <bool kF32Out>
__device__ __forceinline__ void ple_store_word(uint32_t w, uint32_t sb, void* __restrict__ out, size_t j) {
    if constexpr (!kF32Out) {
        // bf16 out = RNE(q * s).  q * s is exact in f32, so rounding it once to bf16
        // equals one correctly rounded bf16 multiply of the exact operands q and s.
        const uint32_t s2 = sb | (sb << 16);
        uint32_t r[4];
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
            // nibbles pp and pp+4 of the word -> bf16x2 (128 + (n ^ 8)) -> minus 136 = signed q
            uint32_t v;
            asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(v) : "r"(w >> (4 * pp)), "r"(0x000F000Fu), "r"(0x43084308u));
            uint32_t q;
            asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(q) : "r"(v), "r"(0x43084308u));
            asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r[pp]) : "r"(q), "r"(s2));
        }
        // r[pp] holds columns (pp, pp+4) of this word; emit (0,1) (2,3) (4,5) (6,7)
        uint4 ov;
        ov.x = __byte_perm(r[0], r[1], 0x5410);
        ov.y = __byte_perm(r[2], r[3], 0x5410);
        ov.z = __byte_perm(r[0], r[1], 0x7632);
        ov.w = __byte_perm(r[2], r[3], 0x7632);
        reinterpret_cast<uint4*>(out)[j] = ov;
    } else {
        const float s = bf16_bits_to_f32(sb);
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            // ((n ^ 8) | 0x4B000000) as f32 = 2^23 + q + 8
            const uint32_t m = ((w >> (4 * e)) & 0xFu) ^ 0x4B000008u;
            v[e] = (__uint_as_float(m) - 8388616.0f) * s;
        }
        float4* o = reinterpret_cast<float4*>(out) + j * 2;
        o[0] = make_float4(v[0], v[1], v[2], v[3]);
        o[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
}

// kWPR > 0: rows of exactly kWPR words (a multiple of kPleThreads; words_per_row and
// groups_per_row are then ignored).  An out-of-range id gives a zero row and raises the
// device error word.
template <bool kF32Out, int kWPR>
__global__ void __launch_bounds__(kPleThreads) ple_gather_kernel(const uint32_t* __restrict__ packed,
                                                                 const uint16_t* __restrict__ scales,
                                                                 const int32_t* __restrict__ ids, int vocab,
                                                                 int words_per_row, int groups_per_row,
                                                                 void* __restrict__ out, uint32_t* err) {
    extern __shared__ __align__(16) uint16_t s_scales[];  // [groups_per_row]
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x;
    const int id = __ldg(ids + t);
    const bool ok = (unsigned)id < (unsigned)vocab;
    if (!ok && threadIdx.x == 0) raise_error(err, G4_DEVERR_BAD_INDEX);
    const int rid = ok ? id : 0;
    if constexpr (kWPR > 0) {
        static_assert(kWPR % kPleThreads == 0 && kWPR % 32 == 0, "whole words per thread, whole 16-byte scale loads");
        constexpr int kW = kWPR / kPleThreads;
        const uint32_t* prow = packed + (size_t)rid * kWPR;
        if (threadIdx.x < kWPR / 32)
            reinterpret_cast<uint4*>(s_scales)[threadIdx.x] =
                __ldg(reinterpret_cast<const uint4*>(scales + (size_t)rid * (kWPR / 4)) + threadIdx.x);
        uint32_t w[kW];
#pragma unroll
        for (int k = 0; k < kW; ++k) w[k] = __ldg(prow + k * kPleThreads + threadIdx.x);
        __syncthreads();
        const size_t orow = (size_t)t * kWPR;
#pragma unroll
        for (int k = 0; k < kW; ++k) {
            const int j = k * kPleThreads + threadIdx.x;
            ple_store_word<kF32Out>(ok ? w[k] : 0u, ok ? (uint32_t)s_scales[j >> 2] : 0u, out, orow + j);
        }
    } else {
        const uint32_t* prow = packed + (size_t)rid * words_per_row;
        const uint16_t* srow = scales + (size_t)rid * groups_per_row;
        const size_t orow = (size_t)t * words_per_row;
        if (groups_per_row % 8 == 0) {  // the row's scales start on a 16-byte boundary
            for (int i = threadIdx.x; i < groups_per_row / 8; i += kPleThreads)
                reinterpret_cast<uint4*>(s_scales)[i] =
                    ok ? __ldg(reinterpret_cast<const uint4*>(srow) + i) : make_uint4(0u, 0u, 0u, 0u);
        } else {
            for (int i = threadIdx.x; i < groups_per_row; i += kPleThreads) s_scales[i] = ok ? __ldg(srow + i) : 0;
        }
        bool staged = false;
        for (int base = 0; base < words_per_row; base += kPleThreads * kPleWords) {
            uint32_t w[kPleWords];
#pragma unroll
            for (int k = 0; k < kPleWords; ++k) {
                const int j = base + k * kPleThreads + threadIdx.x;
                w[k] = (ok && j < words_per_row) ? __ldg(prow + j) : 0u;
            }
            if (!staged) {  // the scales are in shared memory (uniform branch: the loop is the CTA's)
                __syncthreads();
                staged = true;
            }
#pragma unroll
            for (int k = 0; k < kPleWords; ++k) {
                const int j = base + k * kPleThreads + threadIdx.x;
                if (j < words_per_row) ple_store_word<kF32Out>(w[k], s_scales[j >> 2], out, orow + j);  // 4 words = one group
            }
        }
    }
}

g4_status copy_in(void* dst, const void* src, size_t bytes, int src_on_device, cudaStream_t s) {
    G4_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes,
                                  src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s));
    return G4_OK;
}

}  // namespace

extern "C" {

g4_status g4_ple_table_create(g4_ctx* ctx, const void* packed_u8, const void* scales_bf16,
                              int vocab, int width, int group, int src_on_device,
                              g4_ple_table** out) {
    if (!out) return g4::set_error(G4_ERR_INVALID, "g4_ple_table_create: null out");
    *out = nullptr;
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (vocab <= 0 || width <= 0)
        return g4::set_error(G4_ERR_INVALID, "g4_ple_table_create: bad geometry %d x %d", vocab, width);
    if (group != 32 || width % 32 != 0)
        return g4::set_error(G4_ERR_UNSUPPORTED,
                             "g4_ple_table_create: group %d / width %d (group 32 and width %% 32 == 0 required)",
                             group, width);
    if ((packed_u8 == nullptr) != (scales_bf16 == nullptr))
        return g4::set_error(G4_ERR_INVALID, "g4_ple_table_create: packed and scales must both be given or both NULL");
    g4_ple_table* t = new g4_ple_table();
    t->ctx = ctx;
    t->vocab = vocab;
    t->width = width;
    t->group = group;
    const size_t pbytes = (size_t)vocab * (width / 2), sbytes = (size_t)vocab * (width / group) * 2;
    cudaError_t e = cudaMalloc(&t->packed, pbytes);
    if (e == cudaSuccess) e = cudaMalloc(&t->scales, sbytes);
    if (e != cudaSuccess) {
        cudaFree(t->packed);
        cudaFree(t->scales);
        delete t;
        return g4::cuda_error(e, "g4_ple_table_create: cudaMalloc");
    }
    if (packed_u8) {
        st = copy_in(t->packed, packed_u8, pbytes, src_on_device, ctx->stream);
        if (!st) st = copy_in(t->scales, scales_bf16, sbytes, src_on_device, ctx->stream);
        if (!st && !src_on_device) {
            cudaError_t se = cudaStreamSynchronize(ctx->stream);
            if (se != cudaSuccess) st = g4::cuda_error(se, "g4_ple_table_create: sync");
        }
        if (st) {
            g4_ple_table_destroy(t);
            return st;
        }
    }
    *out = t;
    return G4_OK;
}

g4_status g4_ple_table_upload_rows(g4_ctx* ctx, g4_ple_table* tab, int row_start, int rows,
                                   const void* packed_u8, const void* scales_bf16,
                                   int src_on_device) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!tab || !packed_u8 || !scales_bf16)
        return g4::set_error(G4_ERR_INVALID, "g4_ple_table_upload_rows: null argument");
    if (row_start < 0 || rows < 0 || row_start + rows > tab->vocab)
        return g4::set_error(G4_ERR_RANGE, "g4_ple_table_upload_rows: rows [%d, %d) outside vocab %d",
                             row_start, row_start + rows, tab->vocab);
    const size_t prow = tab->width / 2, srow = (size_t)(tab->width / tab->group) * 2;
    st = copy_in(tab->packed + (size_t)row_start * prow, packed_u8, (size_t)rows * prow, src_on_device,
                 ctx->stream);
    if (st) return st;
    st = copy_in(reinterpret_cast<uint8_t*>(tab->scales) + (size_t)row_start * srow, scales_bf16,
                 (size_t)rows * srow, src_on_device, ctx->stream);
    if (st) return st;
    if (!src_on_device) G4_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
    return G4_OK;
}

g4_status g4_ple_table_destroy(g4_ple_table* tab) {
    if (!tab) return G4_OK;
    if (tab->ctx) cudaSetDevice(tab->ctx->device);
    cudaFree(tab->packed);
    cudaFree(tab->scales);
    delete tab;
    return G4_OK;
}

g4_status g4_ple_gather(g4_ctx* ctx, const g4_ple_table* tab, const int32_t* ids, int T,
                        int ids_on_device, void* out, g4_dtype out_dtype) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!tab) return g4::set_error(G4_ERR_INVALID, "g4_ple_gather: null table");
    if (T < 0) return g4::set_error(G4_ERR_INVALID, "g4_ple_gather: T = %d", T);
    if (T == 0) return G4_OK;
    if (!ids || !out) return g4::set_error(G4_ERR_INVALID, "g4_ple_gather: null ids/out");
    if (out_dtype != G4_F32 && out_dtype != G4_BF16)
        return g4::set_error(G4_ERR_INVALID, "g4_ple_gather: out dtype %d", (int)out_dtype);
    if (reinterpret_cast<uintptr_t>(out) % 16 != 0)
        return g4::set_error(G4_ERR_INVALID, "g4_ple_gather: out must be 16-byte aligned");
    const int32_t* d_ids = ids;
    if (!ids_on_device) {
        // gpu-runtime.js:463-470: integer ids in [0, vocab) or throw
        for (int t = 0; t < T; ++t)
            if (ids[t] < 0 || ids[t] >= tab->vocab)
                return g4::set_error(G4_ERR_RANGE, "PLE token id out of range: %d", ids[t]);
        if (ctx->d_ids_cap < (size_t)T) {
            G4_CHECK_CUDA(cudaStreamSynchronize(ctx->stream));
            cudaFree(ctx->d_ids);
            ctx->d_ids = nullptr;
            ctx->d_ids_cap = 0;
            size_t cap = T < 4096 ? 4096 : (size_t)T;
            G4_CHECK_CUDA(cudaMalloc(&ctx->d_ids, cap * sizeof(int32_t)));
            ctx->d_ids_cap = cap;
        }
        G4_CHECK_CUDA(cudaMemcpyAsync(ctx->d_ids, ids, (size_t)T * sizeof(int32_t),
                                      cudaMemcpyHostToDevice, ctx->stream));
        d_ids = ctx->d_ids;
    }
    const int gpr = tab->width / 32, wpr = tab->width / 8;
    const uint32_t* p = reinterpret_cast<const uint32_t*>(tab->packed);
    const dim3 grid((unsigned)T), block(kPleThreads);
    const size_t smem = ((size_t)gpr * 2 + 15) & ~size_t(15);
    if (smem > 48 * 1024) return g4::set_error(G4_ERR_UNSUPPORTED, "g4_ple_gather: width %d", tab->width);
    const uint16_t* sc = static_cast<const uint16_t*>(tab->scales);
    const bool bf = out_dtype == G4_BF16;
    if (wpr == kPleWidthWords)
        return bf ? g4::launch(ctx, "ple_gather_kernel", ple_gather_kernel<false, kPleWidthWords>, grid, block, smem, 1,
                               p, sc, d_ids, tab->vocab, wpr, gpr, out, ctx->d_err)
                  : g4::launch(ctx, "ple_gather_kernel", ple_gather_kernel<true, kPleWidthWords>, grid, block, smem, 1,
                               p, sc, d_ids, tab->vocab, wpr, gpr, out, ctx->d_err);
    return bf ? g4::launch(ctx, "ple_gather_kernel", ple_gather_kernel<false, 0>, grid, block, smem, 1, p, sc, d_ids,
                           tab->vocab, wpr, gpr, out, ctx->d_err)
              : g4::launch(ctx, "ple_gather_kernel", ple_gather_kernel<true, 0>, grid, block, smem, 1, p, sc, d_ids,
                           tab->vocab, wpr, gpr, out, ctx->d_err);
}

}  // extern "C"
