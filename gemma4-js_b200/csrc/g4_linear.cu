// g4_linear.cu -- W4A16 linear: device re-layout, bit-exact dequant, split-K decode GEMV.
//
// The reference uploads `weight_packed` I32 [N, K/8] and `weight_scale` BF16 [N, K/32]
// unchanged (custom-webgpu/gpu-runtime.js:1385-1392) and runs one WGSL thread per
// output element over all of K (W4_SHADER :1068-1102).  Here g4_linear_create
// re-lays the same bits out once, into the order the kernels consume:
//
//   wfrag: uint4 [N/16][K/64][32 lanes]  (one 512-byte block per 16 rows x 64 columns)
//     lane l = 4g + t holds, for rows r0 = 16*nt + g and r1 = r0 + 8 and the two
//     32-column groups G = 2c, 2c+1, word t of that row-group (columns 32G+8t..+7):
//       {word(r0, 2c, t), word(r1, 2c, t), word(r0, 2c+1, t), word(r1, 2c+1, t)}
//     with the 8 nibbles of each word reordered n0 n2 n4 n6 n1 n3 n5 n7 (low to high),
//     so (w >> 4p) & 0x000F000F yields columns (2p, 2p+1) as a bf16x2 pair.
//   sfrag: uint2 [N/16][K/64][8]: {s(r0,2c), s(r1,2c), s(r0,2c+1), s(r1,2c+1)} for g.
//
// That is exactly the register fragment of mma.m16n8k16 (A = 16 weight rows, B = 8
// activation rows) once the k index inside each group is permuted consistently for
// weights and activations, so every lane loads its operand with one 16-byte load and
// activations with two 16-byte loads.  The same blocks feed the tcgen05 GEMM producer.
#include <cooperative_groups.h>
#include <algorithm>
#include <stdio.h>

#include "g4_common.cuh"
#include "g4_linear.cuh"

namespace cg = cooperative_groups;

namespace {

using namespace g4dev;

__host__ __device__ __forceinline__ uint32_t permute_nibbles(uint32_t w) {
    // nibble i of the input goes to position kPos[i] = {0,4,1,5,2,6,3,7}[i]
    uint32_t o = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int pos = (i >> 1) + ((i & 1) << 2);
        o |= ((w >> (4 * i)) & 0xFu) << (4 * pos);
    }
    return o;
}

__host__ __device__ __forceinline__ uint32_t unpermute_nibble(uint32_t w, int i) {
    const int pos = (i >> 1) + ((i & 1) << 2);
    return (w >> (4 * pos)) & 0xFu;
}

// One thread per (n-tile, 64-column chunk, lane).
__global__ void repack_kernel(const uint32_t* __restrict__ raw, const uint16_t* __restrict__ raw_s,
                              int K, int N, int Kc, int NT, uint4* __restrict__ wfrag,
                              uint2* __restrict__ sfrag) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)NT * Kc * 32) return;
    const int lane = (int)(i & 31);
    const long long blk = i >> 5;
    const int c = (int)(blk % Kc);
    const int nt = (int)(blk / Kc);
    const int g = lane >> 2, t = lane & 3;
    const int groups = K / 32, words = K / 8;
    uint32_t out[4];
    uint16_t sc[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int row = nt * 16 + g + ((q & 1) ? 8 : 0);
        const int G = 2 * c + (q >> 1);
        const bool ok = row < N && G < groups;
        const uint32_t wv = ok ? raw[(size_t)row * words + G * 4 + t] : 0x88888888u;
        out[q] = permute_nibbles(wv);
        sc[q] = ok ? raw_s[(size_t)row * groups + G] : (uint16_t)0;
    }
    wfrag[i] = make_uint4(out[0], out[1], out[2], out[3]);
    if (t == 0)
        sfrag[blk * 8 + g] = make_uint2((uint32_t)sc[0] | ((uint32_t)sc[1] << 16),
                                        (uint32_t)sc[2] | ((uint32_t)sc[3] << 16));
}

// GEMM layout (g4_linear_dev::tblk): thread i fills row r = i % 128, half h = (i / 128) % 2
// of block b = i / 256 (slab b / Kc, step b % Kc): 16 bytes of nibbles and one scale.
__global__ void repack_tblk_kernel(const uint32_t* __restrict__ raw, const uint16_t* __restrict__ raw_s, int K,
                                   int N, int Kc, int NS, uint8_t* __restrict__ tblk) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)NS * Kc * 256) return;
    const int r = (int)(i & 127), h = (int)((i >> 7) & 1);
    const long long b = i >> 8;
    const int kc = (int)(b % Kc), ws = (int)(b / Kc);
    const int row = ws * 128 + r, G = kc * 2 + h;  // G: group of 32 columns
    const int groups = K / 32, words = K / 8;
    const bool ok = row < N && G < groups;
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = ok ? permute_nibbles(raw[(size_t)row * words + G * 4 + j]) : 0x88888888u;
    uint8_t* blk = tblk + b * g4::kTblkBytes;
    *reinterpret_cast<uint4*>(blk + h * 2048 + r * 16) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint16_t*>(blk + 4096 + h * 256 + r * 2) = ok ? raw_s[(size_t)row * groups + G] : (uint16_t)0;
}

// Reads one original word back out of the fragment layout.
__device__ __forceinline__ void locate(const g4_linear_dev& L, int row, int word, uint32_t& w,
                                       uint32_t& sbits) {
    const int nt = row >> 4, r16 = row & 15, g = r16 & 7, hi = r16 >> 3;
    const int k = word * 8, Gabs = k >> 5, c = Gabs >> 1, G = Gabs & 1, t = (k & 31) >> 3;
    const size_t blk = (size_t)nt * L.Kc + c;
    const uint4 v = L.wfrag[blk * 32 + g * 4 + t];
    const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
    w = vw[G * 2 + hi];
    const uint2 s = L.sfrag[blk * 8 + g];
    const uint32_t sw = G ? s.y : s.x;
    sbits = hi ? (sw >> 16) : (sw & 0xFFFFu);
}

// dequantizeOfficialW4A16Rows (official-w4a16.js:84-96) over the device layout.
template <bool kF32Out>
__global__ void dequant_kernel(g4_linear_dev L, int row_start, int row_count, void* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int words = L.K / 8;
    if (i >= (long long)row_count * words) return;
    const int lr = (int)(i / words), word = (int)(i - (long long)lr * words);
    uint32_t w, sbits;
    locate(L, row_start + lr, word, w, sbits);
    const float s = bf16_bits_to_f32(sbits);
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = (float)((int)unpermute_nibble(w, e) - 8) * s;
    if constexpr (kF32Out) {
        float4* o = reinterpret_cast<float4*>(out) + i * 2;
        o[0] = make_float4(v[0], v[1], v[2], v[3]);
        o[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint4* o = reinterpret_cast<uint4*>(out) + i;
        *o = make_uint4(pack_bf16x2_bits(v[0], v[1]), pack_bf16x2_bits(v[2], v[3]),
                        pack_bf16x2_bits(v[4], v[5]), pack_bf16x2_bits(v[6], v[7]));
    }
}

constexpr int kGemvWarps = 4;
constexpr int kGemvPass = 32;  // 512-byte blocks staged per pass (16 KB of weights)

// Shared-memory plan of one GEMV CTA: P = blocks staged per pass, M activation rows.
//   [0,128) mbarrier | P*512 weight blocks | P*64 scale blocks | M rows of P*128+16 bytes
// The cross-warp partials reuse the weight area once the last pass is consumed.
__host__ __device__ constexpr int gemv_xstride(int P) { return P * 128 + 16; }  // +16: rows not bank-aliased
__host__ __device__ constexpr int gemv_smem_bytes(int P, int M) {
    return 128 + P * 576 + M * gemv_xstride(P) > 128 + 2 * 4 * 32 * 4 * 4 ? 128 + P * 576 + M * gemv_xstride(P)
                                                                         : 128 + 2 * 4 * 32 * 4 * 4;
}

// Split-K decode GEMV (M <= 16).  CTA (nt, s) owns the 16 weight rows of tile nt and
// the s-th slice of their K blocks.  One thread stages the slice's weight blocks,
// scales and activation rows into shared memory with bulk (TMA) copies on one
// mbarrier; the 4 warps then run dequant + mma.m16n8k16 from shared memory.  Partials
// are summed across warps in shared memory and across the S CTAs of the cluster
// through distributed shared memory: no global scratch, no atomics.
// kNB = number of 8-row activation tiles (1: M <= 8, 2: M <= 16).
// kGeglu (one K slice, one pass): a gate/up linear whose 128-row slabs are 64 gate rows then
// the 64 matching up rows; CTA y computes gate tile 8 (y / 4) + y % 4 and its up tile 4 tiles
// later from one staging of both, and writes bf16(gelu(gate) * up) (GELU_MUL) to y [M, N/2]:
// the GeGLU of the gate/up linear without an f32 round trip and a second launch.
template <int kNB, bool kGeglu>
__global__ void __launch_bounds__(kGemvWarps * 32)
gemv_w4a16_kernel(g4_linear_dev L, const uint16_t* __restrict__ x, int M, int ldx,
                  void* __restrict__ y, int ldy, int y_f32, int chunks_per_split, const float* __restrict__ ple,
                  int ple_ld, uint32_t* err) {
    constexpr int kT = kGeglu ? 2 : 1;  // weight tiles per CTA
    extern __shared__ __align__(128) uint8_t sm[];
    const int P = min(chunks_per_split, kGemvPass);
    const int xstride = gemv_xstride(P);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
    uint8_t* wsm = sm + 128;               // [kT][P * 512]
    uint8_t* ssm = wsm + kT * P * 512;     // [kT][P * 64]
    uint8_t* xsm = ssm + kT * P * 64;
    float* red = reinterpret_cast<float*>(wsm);  // [warps][kT][kNB*4][32], after the last pass

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int split = blockIdx.x;
    const int nt = kGeglu ? (int)(blockIdx.y >> 2) * 8 + (int)(blockIdx.y & 3) : (int)blockIdx.y;
    const int c_begin = split * chunks_per_split;
    const int c_end = min(L.Kc, c_begin + chunks_per_split);

    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    // Dependents are released once this grid's predecessor has completed (every thread has
    // passed its wait): the next kernel's CTAs then prefetch their weights while this one
    // computes, and at most two kernels' CTAs share the SMs.  Released at entry, a chain of
    // dependents ran ahead and took the slots this grid still needed (6.4 vs 3.5 us per
    // GEMV); released after the main loop, the next kernel's weight fetch did not overlap.
    if (threadIdx.x != 0) {
        pdl_wait();
        pdl_trigger();
    }

    float acc[kT][kNB][4];
#pragma unroll
    for (int tt = 0; tt < kT; ++tt)
#pragma unroll
        for (int j = 0; j < kNB; ++j) acc[tt][j][0] = acc[tt][j][1] = acc[tt][j][2] = acc[tt][j][3] = 0.f;

    bool ok = true;
    uint32_t phase = 0;
    for (int p0 = c_begin; p0 < c_end && ok; p0 += kGemvPass, phase ^= 1) {
        const int nch = min(kGemvPass, c_end - p0);
        const int k0 = p0 * 64;
        const int klen = min(L.K, (p0 + nch) * 64) - k0;  // valid activation columns
        if (threadIdx.x == 0) {
            const uint32_t bytes = kT * (nch * 512 + nch * 64) + M * klen * 2;
            mbar_arrive_expect_tx(bar, bytes);
#pragma unroll
            for (int tt = 0; tt < kT; ++tt) {  // kGeglu: the up tile sits 4 tiles after the gate tile
                const size_t blk = (size_t)(nt + 4 * tt) * L.Kc + p0;
                bulk_load(wsm + tt * P * 512, L.wfrag + blk * 32, nch * 512, bar);
                bulk_load(ssm + tt * P * 64, L.sfrag + blk * 8, nch * 64, bar);
            }
            if (p0 == c_begin) {  // weights are immutable; activations come from the predecessor
                pdl_wait();
                pdl_trigger();
            }
            for (int b = 0; b < M; ++b)
                bulk_load(xsm + b * xstride, x + (size_t)b * ldx + k0, klen * 2, bar);
        }
        // Zero the activation tail past K inside the last block (K % 64 == 32).
        if (klen < nch * 64)
            for (int i = threadIdx.x; i < M * 32; i += blockDim.x)
                reinterpret_cast<uint16_t*>(xsm + (i >> 5) * xstride)[klen + (i & 31)] = 0;
        ok = mbar_wait(bar, phase, err);
        __syncthreads();
        if (ok) {
            for (int c = warp; c < nch; c += kGemvWarps)
#pragma unroll
            for (int tt = 0; tt < kT; ++tt) {
                const uint4 wv = *reinterpret_cast<const uint4*>(wsm + tt * P * 512 + c * 512 + lane * 16);
                const uint2 sv = *reinterpret_cast<const uint2*>(ssm + tt * P * 64 + c * 64 + g * 8);
                const uint32_t wq[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int G = 0; G < 2; ++G) {
                    const uint32_t w0 = wq[2 * G], w1 = wq[2 * G + 1];
                    const uint32_t a0[4] = {int4pair_to_bf16x2(w0), int4pair_to_bf16x2(w1),
                                            int4pair_to_bf16x2(w0 >> 4), int4pair_to_bf16x2(w1 >> 4)};
                    const uint32_t a1[4] = {int4pair_to_bf16x2(w0 >> 8), int4pair_to_bf16x2(w1 >> 8),
                                            int4pair_to_bf16x2(w0 >> 12), int4pair_to_bf16x2(w1 >> 12)};
                    const uint32_t sw = G ? sv.y : sv.x;
                    const float s_lo = bf16_bits_to_f32(sw & 0xFFFFu), s_hi = bf16_bits_to_f32(sw >> 16);
#pragma unroll
                    for (int j = 0; j < kNB; ++j) {
                        const int b = j * 8 + g;
                        uint4 xg = make_uint4(0, 0, 0, 0);
                        if (b < M)
                            xg = *reinterpret_cast<const uint4*>(xsm + b * xstride +
                                                                 (c * 64 + G * 32 + t * 8) * 2);
                        const uint32_t b0[2] = {xg.x, xg.y}, b1[2] = {xg.z, xg.w};
                        float d[4];
                        const float z[4] = {0.f, 0.f, 0.f, 0.f};
                        mma_bf16_16816(d, a0, b0, z);
                        mma_bf16_16816(d, a1, b1, d);
                        acc[tt][j][0] = fmaf(s_lo, d[0], acc[tt][j][0]);
                        acc[tt][j][1] = fmaf(s_lo, d[1], acc[tt][j][1]);
                        acc[tt][j][2] = fmaf(s_hi, d[2], acc[tt][j][2]);
                        acc[tt][j][3] = fmaf(s_hi, d[3], acc[tt][j][3]);
                    }
                }
            }
        }
        __syncthreads();  // the buffers are refilled by the next pass
    }
    if (threadIdx.x == 0 && c_begin >= c_end) {  // an empty K slice: thread 0 never reached its wait
        pdl_wait();
        pdl_trigger();
    }
    // ple != null: GELU_PLE epilogue, y bf16 = gelu(v) * ple[b * ple_ld + row]; the factors are
    // loaded here, in flight during the reductions (every thread has passed its PDL wait).
    float pf[kNB][4];
    if (!kGeglu && ple && warp == 0 && split == 0) {
#pragma unroll
        for (int j = 0; j < kNB; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = nt * 16 + g + ((e & 2) ? 8 : 0);
                const int b = j * 8 + 2 * t + (e & 1);
                pf[j][e] = (row < L.N && b < M) ? ple[(size_t)b * ple_ld + row] : 0.f;
            }
    }

    // ---- reduce the warps of the CTA ----
#pragma unroll
    for (int tt = 0; tt < kT; ++tt)
#pragma unroll
        for (int j = 0; j < kNB; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) red[((warp * kT + tt) * kNB * 4 + j * 4 + e) * 32 + lane] = acc[tt][j][e];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int q = 0; q < kT * kNB * 4; ++q) {
            float s = red[q * 32 + lane];
#pragma unroll
            for (int w2 = 1; w2 < kGemvWarps; ++w2) s += red[(w2 * kT * kNB * 4 + q) * 32 + lane];
            red[q * 32 + lane] = s;
        }
    }
    if constexpr (kGeglu) {  // one K slice: the CTA holds whole sums
        if (warp != 0) return;
#pragma unroll
        for (int j = 0; j < kNB; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int f = (int)(blockIdx.y >> 2) * 64 + (int)(blockIdx.y & 3) * 16 + g + ((e & 2) ? 8 : 0);
                const int b = j * 8 + 2 * t + (e & 1);
                if (b < M && f < L.N / 2) {
                    const float gate = red[(j * 4 + e) * 32 + lane], up = red[(kNB * 4 + j * 4 + e) * 32 + lane];
                    reinterpret_cast<uint16_t*>(y)[(size_t)b * ldy + f] = (uint16_t)f32_to_bf16_bits(gelu_ref(gate) * up);
                }
            }
        }
        return;
    }
    // ---- reduce the S CTAs of the cluster through distributed shared memory ----
    const int S = gridDim.x;
    if (S > 1) {
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        if (split == 0 && warp == 0) {
#pragma unroll
            for (int q = 0; q < kNB * 4; ++q) {
                float s = red[q * 32 + lane];
                for (int r = 1; r < S; ++r) s += cluster.map_shared_rank(&red[q * 32 + lane], r)[0];
                red[q * 32 + lane] = s;
            }
        }
        cluster.sync();
        if (split != 0) return;
    }
    if (warp != 0) return;
#pragma unroll
    for (int j = 0; j < kNB; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = nt * 16 + g + ((e & 2) ? 8 : 0);
            const int b = j * 8 + 2 * t + (e & 1);
            if (row < L.N && b < M) {
                const float v = red[(j * 4 + e) * 32 + lane];
                if (ple)
                    reinterpret_cast<uint16_t*>(y)[(size_t)b * ldy + row] =
                        (uint16_t)f32_to_bf16_bits(gelu_ref(v) * pf[j][e]);
                else if (y_f32)
                    reinterpret_cast<float*>(y)[(size_t)b * ldy + row] = v;
                else
                    reinterpret_cast<uint16_t*>(y)[(size_t)b * ldy + row] = (uint16_t)f32_to_bf16_bits(v);
            }
        }
    }
}

}  // namespace

namespace g4 {

g4_status launch_gemv(g4_ctx* ctx, const g4_linear* lin, const uint16_t* x, int M, void* y,
                      int y_f32, const float* ple, int ple_ld) {
    const g4_linear_dev& L = lin->dev;
    static std::atomic<uint64_t> attr_set{0};
    if (!(attr_set.load() & (1ull << ctx->device))) {
        G4_CHECK_CUDA(cudaFuncSetAttribute(gemv_w4a16_kernel<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           gemv_smem_bytes(kGemvPass, 8)));
        G4_CHECK_CUDA(cudaFuncSetAttribute(gemv_w4a16_kernel<2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           gemv_smem_bytes(kGemvPass, 16)));
        attr_set.fetch_or(1ull << ctx->device);
    }
    // Split K over a cluster until there are ~2 CTAs per SM, but only while each CTA keeps
    // >= 24 blocks (1536 columns): a decode GEMV is latency-bound, and the cluster's
    // DSMEM reduction costs more than a short K slice saves (measured at K <= 2048).
    int S = 1;
    while (S < 8 && ((L.NT * S < 2 * ctx->num_sms && (L.Kc + 2 * S - 1) / (2 * S) >= 24) ||
                     (L.Kc + S - 1) / S > kGemvPass))
        S *= 2;
    const int cps = (L.Kc + S - 1) / S;
    for (int m0 = 0; m0 < M; m0 += 16) {
        const int mm = (M - m0) < 16 ? (M - m0) : 16;
        const size_t smem = gemv_smem_bytes(cps < kGemvPass ? cps : kGemvPass, mm);
        const uint16_t* xs = x + (size_t)m0 * L.K;
        void* ys = y_f32 ? (void*)(reinterpret_cast<float*>(y) + (size_t)m0 * L.N)
                         : (void*)(reinterpret_cast<uint16_t*>(y) + (size_t)m0 * L.N);
        const float* ples = ple ? ple + (size_t)m0 * ple_ld : nullptr;
        // the split-K cluster runs along x: grid (S, NT), CTA (split, tile)
        g4_status st = mm <= 8 ? launch(ctx, "gemv_w4a16_kernel", gemv_w4a16_kernel<1, false>, dim3(S, L.NT), dim3(kGemvWarps * 32),
                                        smem, S, L, xs, mm, L.K, ys, L.N, y_f32, cps, ples, ple_ld, ctx->d_err)
                               : launch(ctx, "gemv_w4a16_kernel", gemv_w4a16_kernel<2, false>, dim3(S, L.NT), dim3(kGemvWarps * 32),
                                        smem, S, L, xs, mm, L.K, ys, L.N, y_f32, cps, ples, ple_ld, ctx->d_err);
        if (st) return st;
    }
    return G4_OK;
}

// GeGLU of a gate/up linear (rows in 64-row gate/up slabs) for M <= 16, when one CTA's K
// range is the whole row (one slice, one pass): gemv_w4a16_kernel<kNB, true>.  Returns
// G4_ERR_UNSUPPORTED (nothing launched) otherwise; the caller then takes the planes path.
g4_status launch_gemv_geglu(g4_ctx* ctx, const g4_linear* lin, const uint16_t* x, int M, uint16_t* out) {
    const g4_linear_dev& L = lin->dev;
    if (L.N % 128 != 0 || L.Kc > kGemvPass || M > 16) return G4_ERR_UNSUPPORTED;
    // the split rule of launch_gemv: a GeGLU CTA needs the whole K, so only where it keeps one slice
    if (L.NT < 2 * ctx->num_sms && (L.Kc + 1) / 2 >= 24) return G4_ERR_UNSUPPORTED;
    static std::atomic<uint64_t> attr_set{0};
    const int P = L.Kc;
    const size_t need1 = 128 + 2 * (size_t)P * 576 + 8 * gemv_xstride(P), need2 = 128 + 2 * (size_t)P * 576 + 16 * gemv_xstride(P);
    const size_t red1 = 128 + (size_t)kGemvWarps * 2 * 4 * 32 * 4, red2 = 128 + (size_t)kGemvWarps * 2 * 8 * 32 * 4;
    if (!(attr_set.load() & (1ull << ctx->device))) {
        G4_CHECK_CUDA(cudaFuncSetAttribute(gemv_w4a16_kernel<1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)std::max<size_t>(128 + 2 * (size_t)kGemvPass * 576 + 8 * gemv_xstride(kGemvPass), red1)));
        G4_CHECK_CUDA(cudaFuncSetAttribute(gemv_w4a16_kernel<2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)std::max<size_t>(128 + 2 * (size_t)kGemvPass * 576 + 16 * gemv_xstride(kGemvPass), red2)));
        attr_set.fetch_or(1ull << ctx->device);
    }
    const dim3 grid(1, (unsigned)(L.NT / 2));
    return M <= 8 ? launch(ctx, "gemv_w4a16_kernel<geglu>", gemv_w4a16_kernel<1, true>, grid, dim3(kGemvWarps * 32),
                           std::max(need1, red1), 1, L, x, M, L.K, out, L.N / 2, 0, L.Kc, nullptr, 0, ctx->d_err)
                  : launch(ctx, "gemv_w4a16_kernel<geglu>", gemv_w4a16_kernel<2, true>, grid, dim3(kGemvWarps * 32),
                           std::max(need2, red2), 1, L, x, M, L.K, out, L.N / 2, 0, L.Kc, nullptr, 0, ctx->d_err);
}

}  // namespace g4

extern "C" {

g4_status g4_linear_create(g4_ctx* ctx, const void* packed_i32, const void* scales_bf16, int K,
                           int N, int group, int src_on_device, g4_linear** out) {
    if (!out) return g4::set_error(G4_ERR_INVALID, "g4_linear_create: null out");
    *out = nullptr;
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!packed_i32 || !scales_bf16) return g4::set_error(G4_ERR_INVALID, "g4_linear_create: null weights");
    if (K <= 0 || N <= 0) return g4::set_error(G4_ERR_INVALID, "g4_linear_create: K=%d N=%d", K, N);
    // official-w4a16.js:59-64
    if (K % 8 != 0) return g4::set_error(G4_ERR_INVALID, "inDim must be divisible by 8.");
    if (group <= 0 || K % group != 0) return g4::set_error(G4_ERR_INVALID, "inDim must be divisible by groupSize.");
    if (group != 32)
        return g4::set_error(G4_ERR_UNSUPPORTED, "g4_linear_create: group size %d (only 32 is implemented)", group);
    g4_linear* lin = new g4_linear();
    lin->ctx = ctx;
    g4_linear_dev& L = lin->dev;
    L.K = K;
    L.N = N;
    L.Kc = (K + 63) / 64;
    L.NT = (N + 15) / 16;
    L.NS = (N + 127) / 128;
    const size_t raw_w = (size_t)N * (K / 8) * 4, raw_s = (size_t)N * (K / 32) * 2;
    const size_t nblk = (size_t)L.NT * L.Kc;
    void *dw = nullptr, *ds = nullptr;
    cudaError_t e = cudaMalloc(&L.wfrag, nblk * 32 * sizeof(uint4));
    if (e == cudaSuccess) e = cudaMalloc(&L.sfrag, nblk * 8 * sizeof(uint2));
    if (e == cudaSuccess) e = cudaMalloc(&L.tblk, (size_t)L.NS * L.Kc * g4::kTblkBytes);
    if (e == cudaSuccess && !src_on_device) {
        e = cudaMalloc(&dw, raw_w);
        if (e == cudaSuccess) e = cudaMalloc(&ds, raw_s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(dw, packed_i32, raw_w, cudaMemcpyHostToDevice, ctx->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(ds, scales_bf16, raw_s, cudaMemcpyHostToDevice, ctx->stream);
    }
    if (e == cudaSuccess) {
        const uint32_t* rw = static_cast<const uint32_t*>(src_on_device ? packed_i32 : dw);
        const uint16_t* rs = static_cast<const uint16_t*>(src_on_device ? scales_bf16 : ds);
        const long long threads = (long long)nblk * 32;
        repack_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, ctx->stream>>>(rw, rs, K, N, L.Kc, L.NT,
                                                                                  L.wfrag, L.sfrag);
        e = cudaGetLastError();
        g4::count_launch();
        const long long tthreads = (long long)L.NS * L.Kc * 256;
        if (e == cudaSuccess) {
            repack_tblk_kernel<<<(unsigned)((tthreads + 255) / 256), 256, 0, ctx->stream>>>(rw, rs, K, N, L.Kc, L.NS,
                                                                                           L.tblk);
            e = cudaGetLastError();
            g4::count_launch();
        }
    }
    if (e == cudaSuccess && !src_on_device) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(dw);
    cudaFree(ds);
    if (e != cudaSuccess) {
        g4_linear_destroy(lin);
        return g4::cuda_error(e, "g4_linear_create");
    }
    *out = lin;
    return G4_OK;
}

g4_status g4_linear_destroy(g4_linear* lin) {
    if (!lin) return G4_OK;
    if (lin->ctx) cudaSetDevice(lin->ctx->device);
    cudaFree(lin->dev.wfrag);
    cudaFree(lin->dev.sfrag);
    cudaFree(lin->dev.tblk);
    delete lin;
    return G4_OK;
}

g4_status g4_linear_shape(const g4_linear* lin, int* K, int* N) {
    if (!lin) return g4::set_error(G4_ERR_INVALID, "null linear");
    if (K) *K = lin->dev.K;
    if (N) *N = lin->dev.N;
    return G4_OK;
}

g4_status g4_linear_dequant(g4_ctx* ctx, const g4_linear* lin, int row_start, int row_count,
                            void* out, g4_dtype out_dtype) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!lin || !out) return g4::set_error(G4_ERR_INVALID, "g4_linear_dequant: null argument");
    if (row_start < 0 || row_count < 0 || row_start + row_count > lin->dev.N)
        return g4::set_error(G4_ERR_RANGE, "g4_linear_dequant: rows [%d,%d) outside %d", row_start,
                             row_start + row_count, lin->dev.N);
    if (row_count == 0) return G4_OK;
    const long long threads = (long long)row_count * (lin->dev.K / 8);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    if (out_dtype == G4_F32)
        dequant_kernel<true><<<blocks, 256, 0, ctx->stream>>>(lin->dev, row_start, row_count, out);
    else if (out_dtype == G4_BF16)
        dequant_kernel<false><<<blocks, 256, 0, ctx->stream>>>(lin->dev, row_start, row_count, out);
    else
        return g4::set_error(G4_ERR_INVALID, "g4_linear_dequant: dtype %d", (int)out_dtype);
    G4_CHECK_LAUNCH("dequant_kernel");
    return G4_OK;
}

g4_status g4_linear_w4a16_impl(g4_ctx* ctx, const g4_linear* lin, const void* x_bf16, int M,
                               void* y, g4_dtype y_dtype, int impl) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!lin) return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16: null linear");
    if (M < 0) return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16: M = %d", M);
    if (M == 0) return G4_OK;
    if (!x_bf16 || !y) return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16: null x/y");
    if (y_dtype != G4_F32 && y_dtype != G4_BF16)
        return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16: y dtype %d", (int)y_dtype);
    if (reinterpret_cast<uintptr_t>(x_bf16) % 16 != 0)
        return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16: x must be 16-byte aligned");
    const int y_f32 = y_dtype == G4_F32;
    if (impl == 0) impl = (M <= 16) ? 1 : 2;
    if (impl == 2 && !g4::gemm_supported(lin, M)) impl = 1;
    if (impl == 1) return g4::launch_gemv(ctx, lin, static_cast<const uint16_t*>(x_bf16), M, y, y_f32, nullptr, 0);
    if (impl == 2) return g4::launch_gemm(ctx, lin, static_cast<const uint16_t*>(x_bf16), M, y, y_f32);
    return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16_impl: impl %d", impl);
}

g4_status g4_linear_w4a16(g4_ctx* ctx, const g4_linear* lin, const void* x_bf16, int M, void* y,
                          g4_dtype y_dtype) {
    return g4_linear_w4a16_impl(ctx, lin, x_bf16, M, y, y_dtype, 0);
}

g4_status g4_linear_w4a16_geglu(g4_ctx* ctx, const g4_linear* lin, const void* x_bf16, int M, void* out_bf16) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!lin || !x_bf16 || !out_bf16 || M < 0) return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16_geglu: bad arguments");
    if (lin->dev.N % 128 != 0)
        return g4::set_error(G4_ERR_UNSUPPORTED, "g4_linear_w4a16_geglu: N = %d (whole 128-row slabs)", lin->dev.N);
    if (M == 0) return G4_OK;
    if (reinterpret_cast<uintptr_t>(x_bf16) % 16 != 0)
        return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16_geglu: x must be 16-byte aligned");
    const uint16_t* x = static_cast<const uint16_t*>(x_bf16);
    uint16_t* out = static_cast<uint16_t*>(out_bf16);
    if (M > 16 && g4::gemm_supported(lin, M)) return g4::launch_gemm_geglu(ctx, lin, x, M, out);
    if (M <= 16) {
        st = g4::launch_gemv_geglu(ctx, lin, x, M, out);
        if (st != G4_ERR_UNSUPPORTED) return st;
    }
    g4_planes pl;
    st = g4_linear_w4a16_planes(ctx, lin, x_bf16, M, &pl);
    if (st) return st;
    return g4::launch_geglu_planes(ctx, pl, M, lin->dev.N, out);
}

g4_status g4_linear_w4a16_gelu_ple(g4_ctx* ctx, const g4_linear* lin, const void* x_bf16, int M,
                                   const float* per_layer, int layer, int layers, void* out_bf16) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!lin || !x_bf16 || !per_layer || !out_bf16 || M < 0 || layer < 0 || layer >= layers)
        return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16_gelu_ple: bad arguments");
    if (M == 0) return G4_OK;
    if (reinterpret_cast<uintptr_t>(x_bf16) % 16 != 0)
        return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16_gelu_ple: x must be 16-byte aligned");
    const int N = lin->dev.N;
    if (M <= 16 || !g4::gemm_supported(lin, M))  // GELU_PLE in the GEMV's epilogue
        return g4::launch_gemv(ctx, lin, static_cast<const uint16_t*>(x_bf16), M, out_bf16, 0,
                               per_layer + (size_t)layer * N, layers * N);
    g4_planes pl;
    st = g4_linear_w4a16_planes(ctx, lin, x_bf16, M, &pl);
    if (st) return st;
    return g4_gelu_ple_planes(ctx, &pl, per_layer, layer, layers, N, M, out_bf16);
}

g4_status g4_linear_w4a16_planes(g4_ctx* ctx, const g4_linear* lin, const void* x_bf16, int M, g4_planes* out) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!lin || !out || !x_bf16 || M <= 0) return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16_planes: bad arguments");
    if (reinterpret_cast<uintptr_t>(x_bf16) % 16 != 0)
        return g4::set_error(G4_ERR_INVALID, "g4_linear_w4a16_planes: x must be 16-byte aligned");
    const uint16_t* x = static_cast<const uint16_t*>(x_bf16);
    if (M > 16 && g4::gemm_supported(lin, M)) return g4::launch_gemm_planes(ctx, lin, x, M, out);
    // the GEMV's f32 output is the one plane
    st = g4::ensure_workspace(ctx, (size_t)M * lin->dev.N * 4);
    if (st) return st;
    *out = g4_planes{static_cast<const float*>(ctx->ws), 1, 0, lin->dev.N};
    return g4::launch_gemv(ctx, lin, x, M, ctx->ws, 1, nullptr, 0);
}

}  // extern "C"
