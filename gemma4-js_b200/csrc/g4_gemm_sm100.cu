// g4_gemm_sm100.cu -- W4A16 prefill GEMM on the 5th-generation tensor cores (tcgen05).
//
// Y[M, N] = X[M, K] . dequant(W)[N, K]^T, X bf16, FP32 accumulation in TMEM, Y bf16/f32.
// Replaces GPUOps.w4 for many rows (custom-webgpu/gpu-runtime.js:1316-1324; the
// reference runs one WGSL thread per output over all of K, W4_SHADER :1068-1102).
//
// One CTA computes a 128 x 256 tile of Y:
//   warp 0      TMA producer: X tile [128 x 64] (128B swizzle, the UMMA K-major
//               canonical layout) + the tile's 16 int4 weight blocks (16 x 512 B)
//               + their scales (16 x 64 B) into a 4-stage ring.
//   warp 1      TMEM allocator and MMA issuer: one thread issues tcgen05.mma
//               (M = 128, N = 256, K = 16) x 4 per 64-column step into a 256-column
//               FP32 accumulator in TMEM, and tcgen05.commit frees the stages.
//   warps 2..9  dequant producers: int4 -> bf16 (exact q, times the bf16 scale with one
//               rounding: the compressed-tensors bf16 materialisation, roundFloat32ToBF16
//               of q*s, official-w4a16.js:34-48, :95) written straight into the swizzled
//               K-major B operand, 2 stages; then the epilogue: tcgen05.ld of their TMEM
//               lane quarter, convert, store.
// Every wait is bounded; a timeout raises the context's device error word and the
// kernel winds down (TMEM is always freed).
#include <cooperative_groups.h>
#include <stdio.h>

#include "g4_linear.cuh"
#include "g4_tcgen05.cuh"

namespace cg = cooperative_groups;

namespace {

using namespace g4dev;

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kStages = 4;      // X (+ raw weight, or bf16 B) ring
constexpr int kBStages = 2;     // dequantised B ring (W4 path)
constexpr int kDqWarps = 8;
constexpr int kThreads = (2 + kDqWarps) * 32;
constexpr int kABytes = BM * BK * 2;           // 16 KB
constexpr int kRawBytes = (BN / 16) * 512;      // 8 KB
constexpr int kScBytes = (BN / 16) * 64;        // 1 KB
constexpr int kBBytes = BN * BK * 2;            // 32 KB
constexpr int kTmemCols = 256;
constexpr int kRedPitch = BN + 4;  // floats per row of a parked partial tile (bank-skewed)

// Shared-memory plan.  W4 path: [A x4][B x2][raw x4][scales x4][barriers];
// bf16 path (B loaded by TMA, no dequant): [A x4][B x4][barriers].
template <bool kW4>
struct GemmSmem {
    static constexpr int kBSt = kW4 ? kBStages : kStages;
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + kStages * kABytes;
    static constexpr int kOffRaw = kOffB + kBSt * kBBytes;
    static constexpr int kOffSc = kOffRaw + (kW4 ? kStages * kRawBytes : 0);
    static constexpr int kOffBar = kOffSc + (kW4 ? kStages * kScBytes : 0);
    static constexpr int kBytes = kOffBar + 256 + 1024;  // + alignment slack
};

// Instruction descriptor: D f32, A = B = bf16, both K-major, M = 128, N = 256.
constexpr uint32_t kIdesc = mma_idesc_bf16(BM, BN);

struct GemmParams {
    void* y;
    int M, N, K, ldy, y_f32, ktiles;
    int ksplit;  // CTAs of a cluster that share one output tile, each over 1/ksplit of K
    uint32_t* err;
};

// Split-K reduction of one cluster rank: rows kslice, kslice + S, ... of the tile are
// summed over the S parked partials in rank order (deterministic) and stored.  Thread t
// owns 4 columns of every 4th of those rows; all S x RB loads of a batch of RB rows are
// issued before any is used, so a batch costs one distributed-shared-memory round trip.
template <int S>
__device__ __forceinline__ void split_reduce(uint8_t* smem, cg::cluster_group& cluster, int kslice, int mb, int nb,
                                             int t, const GemmParams& p) {
    constexpr int J = (BM + 4 * S - 1) / (4 * S);  // rows per thread
    constexpr int RB = (16 / S) > 0 ? (16 / S) : 1; // rows per batch
    const int c4 = (t & 63) * 4, rsub = t >> 6;
    const int n = nb * BN + c4;
    const float* peer[S];
#pragma unroll
    for (int r = 0; r < S; ++r) peer[r] = cluster.map_shared_rank(reinterpret_cast<float*>(smem), r);
#pragma unroll
    for (int j0 = 0; j0 < J; j0 += RB) {
        float4 v[RB][S];
#pragma unroll
        for (int jb = 0; jb < RB; ++jb) {
            const int rr = kslice + S * (rsub + 4 * (j0 + jb));
            const bool live = j0 + jb < J && rr < BM && mb * BM + rr < p.M;  // rows past M are not moved
#pragma unroll
            for (int r = 0; r < S; ++r)
                v[jb][r] = live ? *reinterpret_cast<const float4*>(peer[r] + rr * kRedPitch + c4)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int jb = 0; jb < RB; ++jb) {
            const int rr = kslice + S * (rsub + 4 * (j0 + jb));
            if (j0 + jb >= J || rr >= BM) continue;
            float4 acc = v[jb][0];
#pragma unroll
            for (int r = 1; r < S; ++r) {
                acc.x += v[jb][r].x;
                acc.y += v[jb][r].y;
                acc.z += v[jb][r].z;
                acc.w += v[jb][r].w;
            }
            const int row = mb * BM + rr;
            if (row < p.M && n < p.N) {  // N % 8 == 0: the 4 columns are all in or all out
                if (p.y_f32) {
                    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.y) + (size_t)row * p.ldy + n) = acc;
                } else {
                    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
                    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p.y) + (size_t)row * p.ldy + n) =
                        make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
                }
            }
        }
    }
}

// kW4 = true: B = dequant(int4 blocks) by the producer warps (wmap / smap = weight
// blocks / scales).  kW4 = false: B is a bf16 [N, K] matrix loaded by TMA (wmap,
// 128B swizzle), e.g. the tied bf16 LM head; smap is unused.
template <bool kW4>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                    const __grid_constant__ CUtensorMap smap, GemmParams p) {
    using L = GemmSmem<kW4>;
    constexpr int kOffA = L::kOffA, kOffB = L::kOffB, kOffRaw = L::kOffRaw, kOffSc = L::kOffSc, kOffBar = L::kOffBar;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // Offset the __shared__ array itself (not an integer round trip) so the compiler keeps
    // shared-memory addressing for every access through `smem`.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* load_full = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* load_empty = load_full + kStages;
    uint64_t* b_full = load_empty + kStages;
    uint64_t* b_empty = b_full + kBStages;
    uint64_t* acc_full = b_empty + kBStages;
    uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.ksplit;
    const int mb = blockIdx.x / S, kslice = blockIdx.x % S, nb = blockIdx.y;
    // this CTA's k-tiles: [k0, k0 + KT)
    const int per = (p.ktiles + S - 1) / S;
    const int k0 = kslice * per;
    const int KT = max(0, min(p.ktiles, k0 + per) - k0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&load_full[s], 1);
            mbar_init(&load_empty[s], kW4 ? 1 + kDqWarps : 1);
        }
        for (int s = 0; s < kBStages; ++s) {
            mbar_init(&b_full[s], kDqWarps);
            mbar_init(&b_empty[s], 1);
        }
        mbar_init(acc_full, 1);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_base_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_base_slot;
    pdl_trigger();
    if (!(warp == 0 && lane == 0)) pdl_wait();  // the TMA thread waits after prefetching weights

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tensor_map(&xmap);
            prefetch_tensor_map(&wmap);
            if (kW4) prefetch_tensor_map(&smap);
            // Weights are immutable: start the first stages' weight copies before waiting for
            // the predecessor kernel that produces X.
            const int pre = KT < kStages ? KT : kStages;
            for (int i = 0; i < pre; ++i) {
                const int kt = k0 + i;
                if constexpr (kW4) {
                    mbar_arrive_expect_tx(&load_full[i], kABytes + kRawBytes + kScBytes);
                    tma_load_2d(smem + kOffRaw + i * kRawBytes, &wmap, &load_full[i], kt * 128, nb * (BN / 16));
                    tma_load_2d(smem + kOffSc + i * kScBytes, &smap, &load_full[i], kt * 16, nb * (BN / 16));
                } else {
                    mbar_arrive_expect_tx(&load_full[i], kABytes + kBBytes);
                    tma_load_2d(smem + kOffB + i * kBBytes, &wmap, &load_full[i], kt * BK, nb * BN);
                }
            }
            pdl_wait();
            for (int i = 0; i < pre; ++i)
                tma_load_2d(smem + kOffA + i * kABytes, &xmap, &load_full[i], (k0 + i) * BK, mb * BM);
            int issued = pre;
            for (int i = pre; i < KT; ++i) {
                const int s = i % kStages, kt = k0 + i;
                if (i >= kStages && !mbar_wait(&load_empty[s], ((i / kStages) - 1) & 1, p.err)) break;
                if constexpr (kW4) {
                    mbar_arrive_expect_tx(&load_full[s], kABytes + kRawBytes + kScBytes);
                    tma_load_2d(smem + kOffA + s * kABytes, &xmap, &load_full[s], kt * BK, mb * BM);
                    tma_load_2d(smem + kOffRaw + s * kRawBytes, &wmap, &load_full[s], kt * 128, nb * (BN / 16));
                    tma_load_2d(smem + kOffSc + s * kScBytes, &smap, &load_full[s], kt * 16, nb * (BN / 16));
                } else {
                    mbar_arrive_expect_tx(&load_full[s], kABytes + kBBytes);
                    tma_load_2d(smem + kOffA + s * kABytes, &xmap, &load_full[s], kt * BK, mb * BM);
                    tma_load_2d(smem + kOffB + s * kBBytes, &wmap, &load_full[s], kt * BK, nb * BN);
                }
                issued = i + 1;
            }
            // Drain: our copies must land before the CTA can exit.
            for (int i = issued > kStages ? issued - kStages : 0; i < issued; ++i)
                mbar_wait(&load_full[i % kStages], (i / kStages) & 1, p.err);
        }
    } else if (warp == 1) {
        // -------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            bool ok = true;
            for (int i = 0; i < KT && ok; ++i) {
                const int s = i % kStages, sb = kW4 ? i % kBStages : s;
                ok = mbar_wait(&load_full[s], (i / kStages) & 1, p.err);
                if (kW4 && ok) ok = mbar_wait(&b_full[sb], (i / kBStages) & 1, p.err);
                if (!ok) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(smem + kOffA + s * kABytes);
                const uint32_t b0 = smem_u32(smem + kOffB + sb * kBBytes);
#pragma unroll
                for (int ks = 0; ks < BK / 16; ++ks)
                    tc_mma_ss(tmem, sw128_desc(a0 + ks * 32), sw128_desc(b0 + ks * 32), kIdesc,
                                (i > 0 || ks > 0) ? 1u : 0u);
                tc_commit(&load_empty[s]);        // X (and bf16 B) stage consumed
                if (kW4) tc_commit(&b_empty[sb]);  // dequantised B stage consumed
            }
            tc_commit(acc_full);  // accumulator complete (or abandoned after a timeout)
        }
    } else {
        // ----------------------------------------------------- dequant producers
        const int wd = warp - 2;  // 0..7: n-tiles 2wd, 2wd+1 of this CTA's 16
        const int g = lane >> 2, t = lane & 3;
        bool ok = true;
        for (int i = 0; kW4 && i < KT && ok; ++i) {
            const int s = i % kStages, sb = i % kBStages;
            ok = mbar_wait_warp(&load_full[s], (i / kStages) & 1, p.err);
            if (ok && i >= kBStages) ok = mbar_wait_warp(&b_empty[sb], ((i / kBStages) - 1) & 1, p.err);
            if (!ok) break;
            const uint8_t* raw = smem + kOffRaw + s * kRawBytes;
            const uint8_t* sc = smem + kOffSc + s * kScBytes;
            uint8_t* bt = smem + kOffB + sb * kBBytes;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int j = 2 * wd + e;
                const uint4 wv = *reinterpret_cast<const uint4*>(raw + j * 512 + lane * 16);
                const uint2 sv = *reinterpret_cast<const uint2*>(sc + j * 64 + g * 8);
                const uint32_t wq[4] = {wv.x, wv.y, wv.z, wv.w};  // (r0,G0) (r1,G0) (r0,G1) (r1,G1)
                const uint32_t sq[4] = {__byte_perm(sv.x, 0, 0x1010), __byte_perm(sv.x, 0, 0x3232),
                                        __byte_perm(sv.y, 0, 0x1010), __byte_perm(sv.y, 0, 0x3232)};
#pragma unroll
                for (int qq = 0; qq < 4; ++qq) {
                    // odd rows take the other group first: the 8 lanes of a store phase then
                    // cover 8 distinct 16-byte bank groups
                    const bool odd = g & 1;
                    const int q = odd ? (qq ^ 2) : qq;
                    const int hi = q & 1, G = q >> 1;
                    const uint32_t wsel = odd ? wq[qq ^ 2] : wq[qq];  // static indices: stays in registers
                    const uint32_t ssel = odd ? sq[qq ^ 2] : sq[qq];
                    uint32_t o[4];
#pragma unroll
                    for (int pp = 0; pp < 4; ++pp) {
                        const uint32_t qv = int4pair_to_bf16x2(wsel >> (4 * pp));
                        asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(o[pp]) : "r"(qv), "r"(ssel));
                    }
                    const int n = 16 * j + g + 8 * hi;  // row of the B tile
                    const int c16 = 4 * G + t;          // 16-byte chunk along K
                    uint8_t* dst = bt + (n >> 3) * 1024 + (n & 7) * 128 + ((c16 ^ (n & 7)) << 4);
                    *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
                }
            }
            fence_proxy_async_smem();  // make the generic stores visible to the tensor core
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&b_full[sb]);
                mbar_arrive(&load_empty[s]);
            }
        }
        // ------------------------------------------------------------- epilogue
        if (S > 1) {
            // Split K: park this CTA's FP32 partial tile in its (now idle) shared memory;
            // the cluster sums the S partials below.
            const bool row_live = mb * BM + (warp & 3) * 32 + lane < p.M;  // rows past M are never read
            if (KT == 0) {  // an empty K slice contributes zeros (its accumulator was never written)
                const int quarter = warp & 3, col0 = (warp < 6) ? 0 : 128;
                float* red = reinterpret_cast<float*>(smem) + (quarter * 32 + lane) * kRedPitch + col0;
                if (row_live)
                    for (int c = 0; c < 128; c += 4) *reinterpret_cast<uint4*>(red + c) = make_uint4(0, 0, 0, 0);
            } else if (mbar_wait_warp(acc_full, 0, p.err)) {
                tc_fence_after();
                const int quarter = warp & 3, col0 = (warp < 6) ? 0 : 128;
                float* red = reinterpret_cast<float*>(smem) + (quarter * 32 + lane) * kRedPitch + col0;
#pragma unroll 1
                for (int c = 0; c < 128; c += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(col0 + c), r);
                    tmem_ld_wait(r);
                    if (row_live) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<uint4*>(red + c + i) = make_uint4(r[i], r[i + 1], r[i + 2], r[i + 3]);
                    }
                }
            }
        } else if (mbar_wait_warp(acc_full, 0, p.err)) {
            tc_fence_after();
            const int quarter = warp & 3;          // TMEM lanes 32*quarter .. +31
            const int col0 = (warp < 6) ? 0 : 128; // two warps per lane quarter
            const int row = mb * BM + quarter * 32 + lane;
#pragma unroll 1
            for (int c = 0; c < 128; c += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(col0 + c), r);
                tmem_ld_wait(r);
                const int n0 = nb * BN + col0 + c;
                if (row < p.M && n0 < p.N) {
                    if (p.y_f32) {
                        float* yr = reinterpret_cast<float*>(p.y) + (size_t)row * p.ldy + n0;
                        if (n0 + 32 <= p.N) {
#pragma unroll
                            for (int i = 0; i < 32; i += 4)
                                *reinterpret_cast<uint4*>(yr + i) = make_uint4(r[i], r[i + 1], r[i + 2], r[i + 3]);
                        } else {
                            const int lim = p.N - n0;
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (i < lim) yr[i] = __uint_as_float(r[i]);
                        }
                    } else {
                        uint16_t* yr = reinterpret_cast<uint16_t*>(p.y) + (size_t)row * p.ldy + n0;
                        uint32_t h[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
                            h[i] = *reinterpret_cast<uint32_t*>(&b2);
                        }
                        if (n0 + 32 <= p.N) {
#pragma unroll
                            for (int i = 0; i < 16; i += 4)
                                *reinterpret_cast<uint4*>(yr + 2 * i) = make_uint4(h[i], h[i + 1], h[i + 2], h[i + 3]);
                        } else {
                            const int lim = p.N - n0;
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (i < lim) yr[i] = (uint16_t)(h[i >> 1] >> ((i & 1) * 16));
                        }
                    }
                }
            }
        }
    }
    if (S > 1) {
        // Deterministic cluster reduction through distributed shared memory: CTA `kslice`
        // sums rows kslice, kslice + S, ... of the tile over ranks 0..S-1 in order.
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        if (warp >= 2) {
            switch (S) {
                case 2: split_reduce<2>(smem, cluster, kslice, mb, nb, threadIdx.x - 64, p); break;
                case 3: split_reduce<3>(smem, cluster, kslice, mb, nb, threadIdx.x - 64, p); break;
                case 4: split_reduce<4>(smem, cluster, kslice, mb, nb, threadIdx.x - 64, p); break;
                case 5: split_reduce<5>(smem, cluster, kslice, mb, nb, threadIdx.x - 64, p); break;
                case 6: split_reduce<6>(smem, cluster, kslice, mb, nb, threadIdx.x - 64, p); break;
                case 7: split_reduce<7>(smem, cluster, kslice, mb, nb, threadIdx.x - 64, p); break;
                default: split_reduce<8>(smem, cluster, kslice, mb, nb, threadIdx.x - 64, p); break;
            }
        }
        cluster.sync();  // peers may still be reading this CTA's partial
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

namespace g4 {

// Grid: one CTA per 128 x 256 output tile; when that leaves the GPU under-filled, the K
// range of each tile is split over a cluster of up to 8 CTAs (>= 4 k-tiles each) and
// the partials are summed through distributed shared memory.
template <bool kW4>
g4_status launch_tiles(g4_ctx* ctx, const CUtensorMap& xmap, const CUtensorMap& wmap, const CUtensorMap& smap,
                       GemmParams p) {
    static std::atomic<uint64_t> attr_set{0};
    if (!(attr_set.load() & (1ull << ctx->device))) {
        G4_CHECK_CUDA(cudaFuncSetAttribute(gemm_tcgen05_kernel<kW4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           GemmSmem<kW4>::kBytes));
        attr_set.fetch_or(1ull << ctx->device);
    }
    const int mt = (p.M + BM - 1) / BM, nt = (p.N + BN - 1) / BN;
    if (nt > 65535) return set_error(G4_ERR_UNSUPPORTED, "tcgen05 GEMM: N=%d too large", p.N);
    int S = 1;
    while (S < 8 && mt * nt * (S + 1) <= ctx->num_sms && p.ktiles / (S + 1) >= 4) ++S;
    p.ksplit = S;
    return launch(ctx, kW4 ? "gemm_tcgen05_kernel<W4>" : "gemm_tcgen05_kernel<bf16>", gemm_tcgen05_kernel<kW4>,
                  dim3(mt * S, nt), dim3(kThreads), GemmSmem<kW4>::kBytes, S, xmap, wmap, smap, p);
}

bool gemm_supported(const g4_linear* lin, int M) {
    // row pitches of X (K bf16) and Y (N values) must allow 16-byte vector access
    return M >= 1 && lin->dev.K % 32 == 0 && lin->dev.N % 8 == 0;
}

g4_status launch_gemm_bf16(g4_ctx* ctx, const CUtensorMap& bmap, int N, int K, const uint16_t* x, int M,
                           float* y) {
    if (K % 8 != 0 || N % 8 != 0) return set_error(G4_ERR_UNSUPPORTED, "tcgen05 bf16 GEMM: K=%d N=%d", K, N);
    CUtensorMap xmap;
    g4_status st = encode_tensor_map_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, const_cast<uint16_t*>(x), K, M,
                                        (uint64_t)K * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    GemmParams p{};
    p.y = y;
    p.M = M;
    p.N = N;
    p.K = K;
    p.ldy = N;
    p.y_f32 = 1;
    p.ktiles = (K + BK - 1) / BK;
    p.err = ctx->d_err;
    return launch_tiles<false>(ctx, xmap, bmap, bmap, p);
}

}  // namespace g4
