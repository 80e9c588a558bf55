// g4_gemm_w4.cu -- W4A16 GEMM on the tcgen05 tensor cores with the dequantised weights
// held in tensor memory.
//
// Y[M, N] = X[M, K] . dequant(W)[N, K]^T, X bf16, FP32 accumulation in TMEM, Y bf16/f32.
// Replaces GPUOps.w4 for many rows (custom-webgpu/gpu-runtime.js:1316-1324; the
// reference runs one WGSL thread per output over all of K, W4_SHADER :1068-1102).
//
// The tensor core computes tiles of Y^T: D[128 weight rows, T tokens] += Wq[128, 16] .
// X[T, 16]^T, with Wq the A operand read from TMEM and X the B operand read from shared
// memory (128-byte swizzled, K-major, loaded by TMA).  The dequantised weights go from
// registers straight into TMEM (tcgen05.st), so shared memory carries only X and the
// packed int4 blocks: ~73 KB per 128 x 256 x 64 step instead of ~114 KB when the bf16
// weights are staged in shared memory, which is what bounds a one-CTA tile at 128 B per
// clock of shared-memory bandwidth.
//
// Roles (576 threads, one CTA per SM, persistent over tiles when there are enough of them):
//   warp 0       TMA producer: per 128-column stage, X [T x 128] (two 64-column boxes)
//                and the stage's two packed weight blocks (128 rows x 64 int4 + 256 bf16
//                scales each, 9216 B contiguous, one bulk copy) into a 3-stage ring.
//                Weight blocks of the first stages are requested before waiting on the
//                predecessor kernel (programmatic dependent launch): they are immutable.
//   warp 1       TMEM allocator (512 columns: accumulator 0..255, weight ring 256..383)
//                and MMA issuer: one thread, tcgen05.mma M = 128, N = T, K = 16, eight
//                per stage.  tcgen05.mma issue is nearly synchronous with its execution,
//                so each synchronisation point (two barrier waits) covers 8 MMAs.
//   warps 2..9   dequantisers: warp w owns TMEM lane quarter w % 4 (32 weight rows) and
//                one 64-column half of the stage; q = nibble - 8 exactly in bf16, times
//                the bf16 scale with one rounding (the compressed-tensors bf16
//                materialisation, roundFloat32ToBF16 of q*s, official-w4a16.js:34-48,
//                :95), then tcgen05.st into a 2-stage TMEM ring.
//   warps 10..17 epilogue: warp w drains lane quarter w % 4, tokens 128 * ((w - 10) / 4)
//                + 0..127, with tcgen05.ld into registers, into the X stage(s) the tile's
//                last MMAs consumed ([token][128 rows], bf16 or f32), releases the
//                accumulator after its last load, and one thread stores the tile with TMA.
// When the tiles do not fill the GPU, K is split over S CTAs per tile; each stores its
// FP32 partial tile (through the same staged TMA store) into plane `slice` of an
// L2-resident workspace [S][Mp][N], and splitk_sum_kernel adds the planes in slice order
// (deterministic).  Every wait is bounded; a timeout raises the context's device error
// word and the kernel winds down (TMEM is always freed).
#include "g4_linear.cuh"
#include "g4_tcgen05.cuh"

namespace {

using namespace g4dev;

constexpr int TW = 128;     // weight rows per tile (MMA M)
constexpr int TTmax = 256;  // tokens per tile (MMA N), at most
constexpr int TK = 64;      // K per weight block / X box (one 128-byte swizzle row)
constexpr int kSub = 2;     // weight blocks per pipeline stage (K = 128 per stage)
constexpr int kStages = 3;  // X + weight-block ring (shared memory)
constexpr int kAStages = 2; // dequantised weight ring (TMEM, 64 columns each)
constexpr int kDq = 8;
constexpr int kEpi = 8;
constexpr int kThreads = (2 + kDq + kEpi) * 32;
constexpr int kXSub = TTmax * TK * 2;         // 32 KB: one [T x 64] box
constexpr int kXBytes = kSub * kXSub;         // 64 KB per stage
constexpr int kBlkBytes = g4::kTblkBytes;     // 4096 B of nibbles + 512 B of scales
constexpr int kTmemCols = 512;
constexpr int kMaxSlices = 8;  // split-K slices (partial planes) per linear
constexpr int kAccCol = 0, kACol = 256;

struct Smem {
    static constexpr int kOffX = 0;
    static constexpr int kOffBlk = kOffX + kStages * kXBytes;
    static constexpr int kOffBar = kOffBlk + kStages * kSub * kBlkBytes;
    static constexpr int kBytes = kOffBar + 256 + 1024;  // + alignment slack
};
static_assert(TTmax * TW * 2 <= kXBytes && 128 * TW * 4 <= kXBytes, "an output stage must fit in an X stage");
static_assert(Smem::kBytes <= 232448, "shared memory plan exceeds 227 KB");

struct W4Params {
    const uint8_t* tblk;  // [NS][Kc] weight blocks
    void* y;
    int M, N, ldy, y_f32;
    int Kc;          // 64-column weight blocks along K
    int NS, MT, TT;  // weight slabs of 128 rows, token tiles, tokens per tile (multiple of 32)
    int ksplit;      // CTAs sharing one tile, each over a slice of K (1: no split)
    int kper;        // weight blocks per K slice
    float* part;     // ksplit > 1: partial planes [ksplit][Mp][N] f32, Mp = MT * (TT > 128 ? 256 : TT)
    // geglu: the weight rows of every 128-row slab are 64 gate rows then the 64 matching up
    // rows; y is bf16 [M, N/2] = gelu(gate) * up (GELU_MUL), computed from the staged tile.
    int geglu;
    int wsplit;  // weight blocks and X on separate stage barriers (see the kernel)
    uint32_t* err;
};

// GeGLU epilogue (W4Params::geglu): bf16 act[m, 64 ws + f] = gelu(gate_f) * up_f from a staged
// f32 [128 tokens][128 rows] stage; warp (q, e) takes tokens 128e + q, +4, ..., lane l the
// features 2l, 2l + 1 (each store writes one 128-byte row).  Compiled only into the GeGLU
// instance of the kernel, so its
// registers do not add to the plain kernel's (a separate template instance).
__device__ __forceinline__ void geglu_rows(const uint8_t* stage, int q, int e, int lane, int ms, int ws,
                                        const W4Params& p) {
    const int half = TW / 2, ldo = p.N / 2;
    for (int tl = q; tl < 128; tl += 4) {
        const int tok = 128 * e + tl;
        const int m = ms * p.TT + tok;
        if (tok >= p.TT || m >= p.M) break;
        const float2 gt = reinterpret_cast<const float2*>(stage + (size_t)tl * TW * 4)[lane];
        const float2 up = reinterpret_cast<const float2*>(stage + (size_t)tl * TW * 4 + half * 4)[lane];
        reinterpret_cast<uint32_t*>(reinterpret_cast<uint16_t*>(p.y) + (size_t)m * ldo + ws * half)[lane] =
            pack_bf16x2_bits(gelu_ref(gt.x) * up.x, gelu_ref(gt.y) * up.y);
    }
}

template <bool kGeglu>
__global__ void __launch_bounds__(kThreads, 1)
gemm_w4_tmem_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap ymap,
                    const W4Params p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // Offset the __shared__ array itself (not an integer round trip) so the compiler keeps
    // shared-memory addressing for every access through `smem`.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* load_full = reinterpret_cast<uint64_t*>(smem + Smem::kOffBar);
    uint64_t* load_empty = load_full + kStages;
    uint64_t* a_full = load_empty + kStages;
    uint64_t* a_empty = a_full + kAStages;
    uint64_t* acc_full = a_empty + kAStages;
    uint64_t* acc_empty = acc_full + 1;
    // p.wsplit (a grid of at most one tile per CTA, a decode-size linear): the weight blocks
    // of a stage complete on w_full and its X boxes on load_full, so the dequantisers, which
    // need only the blocks (requested before the PDL wait), start while X (the predecessor's
    // output) is still on its way.  Otherwise both arrive on load_full (the persistent
    // prefill GEMM measured 1-2 % faster that way).
    uint64_t* w_full = acc_empty + 1;
    uint64_t* wb = p.wsplit ? w_full : load_full;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(w_full + kStages);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.ksplit;
    const int ntiles = p.NS * p.MT;
    // S == 1: persistent, tiles blockIdx.x, + gridDim.x, ...; S > 1: CTAs t*S .. t*S+S-1 own
    // tile t, each one K slice.
    const int tile0 = S > 1 ? (int)blockIdx.x / S : (int)blockIdx.x;
    const int tstep = S > 1 ? ntiles : (int)gridDim.x;
    const int kslice = S > 1 ? (int)blockIdx.x % S : 0;
    const int k0 = kslice * p.kper;                       // first weight block of this CTA's K range
    const int KT = max(0, min(p.Kc, k0 + p.kper) - k0);   // weight blocks per tile (the host leaves no slice empty)
    const int NST = (KT + kSub - 1) / kSub;            // pipeline stages per tile
    const uint32_t xsub = (uint32_t)p.TT * TK * 2;     // bytes of one X box
    // The output of an unsplit tile leaves through TMA stores staged in the X stages that
    // the tile's last MMAs read (bf16: one stage holds [T][128]; f32: one stage per 128
    // tokens); those stages are handed back to the producer by the epilogue (after the
    // stores have read them) instead of by the MMA commit.
    const bool out_f32 = p.y_f32 || S > 1 || kGeglu;  // partial planes and GeGLU inputs are f32
    const int out_stages = (out_f32 && p.TT > 128) ? 2 : 1;
    const bool staged = NST >= out_stages;
    const int plane_row0 = kslice * p.MT * (p.TT > 128 ? 256 : p.TT);  // first row of this CTA's output plane

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&load_full[s], 1);
            mbar_init(&w_full[s], 1);
            mbar_init(&load_empty[s], 1 + kDq);  // the MMA (X read) and every dequant warp (blocks read)
        }
        for (int s = 0; s < kAStages; ++s) {
            mbar_init(&a_full[s], kDq);
            mbar_init(&a_empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, kEpi);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_trigger();
    // Only the TMA thread (after its weight prefetch) and the epilogue touch memory that a
    // predecessor kernel may still be producing (X) or reading (Y).
    if (warp >= 2 + kDq) pdl_wait();

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tensor_map(&xmap);
            int pre = 0;
            for (int t = tile0; t < ntiles && pre < kStages; t += tstep)
                for (int j = 0; j < NST && pre < kStages; ++j, ++pre) {
                    const int ws = t / p.MT, nsub = min(kSub, KT - j * kSub);
                    mbar_arrive_expect_tx(&wb[pre], (uint32_t)nsub * (kBlkBytes + (p.wsplit ? 0 : xsub)));
                    bulk_load(smem + Smem::kOffBlk + pre * kSub * kBlkBytes,
                              p.tblk + ((size_t)ws * p.Kc + k0 + j * kSub) * kBlkBytes, nsub * kBlkBytes,
                              &wb[pre]);
                }
            pdl_wait();
            bool ok = true;
            int g = 0;
            for (int t = tile0; t < ntiles && ok; t += tstep) {
                const int ws = t / p.MT, ms = t % p.MT;
                for (int j = 0; j < NST; ++j, ++g) {
                    const int s = g % kStages, nsub = min(kSub, KT - j * kSub);
                    if (g >= kStages) {
                        if (!mbar_wait(&load_empty[s], ((g / kStages) - 1) & 1, p.err, 0x101)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&wb[s], (uint32_t)nsub * (kBlkBytes + (p.wsplit ? 0 : xsub)));
                        bulk_load(smem + Smem::kOffBlk + s * kSub * kBlkBytes,
                                  p.tblk + ((size_t)ws * p.Kc + k0 + j * kSub) * kBlkBytes, nsub * kBlkBytes,
                                  &wb[s]);
                    }
                    if (p.wsplit) mbar_arrive_expect_tx(&load_full[s], (uint32_t)nsub * xsub);
                    for (int u = 0; u < nsub; ++u)
                        tma_load_2d(smem + Smem::kOffX + s * kXBytes + u * kXSub, &xmap, &load_full[s],
                                    (k0 + j * kSub + u) * TK, ms * p.TT);
                }
            }
            // Drain: our copies must land before the CTA can exit.
            for (int j = g > kStages ? g - kStages : 0; j < g; ++j)
                mbar_wait(&load_full[j % kStages], (j / kStages) & 1, p.err, 0x102);
            const int gw = g > pre ? g : pre;  // weight blocks requested, prefetched ones included
            if (p.wsplit)
                for (int j = gw > kStages ? gw - kStages : 0; j < gw; ++j)
                    mbar_wait(&w_full[j % kStages], (j / kStages) & 1, p.err, 0x10a);
        }
        __syncwarp();
    } else if (warp == 1) {
        // -------------------------------------------------------------- MMA issuer
        if (lane == 0 && KT > 0) {
            const uint32_t idesc = mma_idesc_bf16(TW, p.TT);
            bool ok = true;
            int g = 0, tj = 0;
            for (int t = tile0; t < ntiles && ok; t += tstep, ++tj) {
                if (tj > 0 && !mbar_wait(acc_empty, (tj - 1) & 1, p.err, 0x103)) break;  // epilogue drained the accumulator
                tc_fence_after();
                for (int j = 0; j < NST; ++j, ++g) {
                    const int s = g % kStages, sa = g % kAStages, nsub = min(kSub, KT - j * kSub);
                    if (!mbar_wait(&load_full[s], (g / kStages) & 1, p.err, 0x104) ||
                        !mbar_wait(&a_full[sa], (g / kAStages) & 1, p.err, 0x105)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t xa = smem_u32(smem + Smem::kOffX + s * kXBytes);
                    const uint32_t aa = tmem + kACol + sa * (kSub * 32);
#pragma unroll
                    for (int u = 0; u < kSub; ++u)
                        if (u < nsub)
#pragma unroll
                            for (int ks = 0; ks < TK / 16; ++ks)
                                tc_mma_ts(tmem + kAccCol, aa + u * 32 + ks * 8, sw128_desc(xa + u * kXSub + ks * 32),
                                          idesc, (j > 0 || u > 0 || ks > 0) ? 1u : 0u);
                    tc_commit(&a_empty[sa]);                                  // weight stage consumed
                    if (!(staged && j >= NST - out_stages)) tc_commit(&load_empty[s]);  // X stage consumed
                }
                tc_commit(acc_full);  // tile complete (or abandoned after a timeout)
            }
        }
        __syncwarp();
    } else if (warp < 2 + kDq) {
        // ---------------------------------------------------------- dequantisers
        const int q = warp & 3, h = (warp - 2) >> 2;  // lane quarter, weight block of the stage
        const int r = 32 * q + lane;                   // weight row of the tile = TMEM lane
        const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + kACol + h * 32;
        bool ok = true;
        int g = 0;
        for (int t = tile0; t < ntiles && ok; t += tstep) {
            for (int j = 0; j < NST; ++j, ++g) {
                const int s = g % kStages, sa = g % kAStages;
                const bool live = h < min(kSub, KT - j * kSub);
                ok = mbar_wait_warp(&wb[s], (g / kStages) & 1, p.err, 0x106);
                if (ok && g >= kAStages) ok = mbar_wait_warp(&a_empty[sa], ((g / kAStages) - 1) & 1, p.err, 0x107);
                if (!ok) break;
                if (live) {
                    const uint8_t* blk = smem + Smem::kOffBlk + (s * kSub + h) * kBlkBytes;
                    uint32_t o[32];
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const uint4 wv = *reinterpret_cast<const uint4*>(blk + half * 2048 + r * 16);
                        const uint32_t sb = *reinterpret_cast<const uint16_t*>(blk + 4096 + half * 256 + r * 2);
                        const uint32_t s2 = sb | (sb << 16);
                        const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                        for (int wi = 0; wi < 4; ++wi)
#pragma unroll
                            for (int pp = 0; pp < 4; ++pp) {
                                // nibble pair pp of word wi = columns 32 half + 8 wi + 2 pp, +1
                                const uint32_t qv = int4pair_to_bf16x2(w[wi] >> (4 * pp));
                                asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(o[half * 16 + wi * 4 + pp]) : "r"(qv), "r"(s2));
                            }
                    }
                    tmem_st_32x32b_x32(ta + sa * (kSub * 32), o);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&load_empty[s]);  // the blocks' registers are consumed above
                if (live) tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_full[sa]);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------- epilogue
        const int q = warp & 3, e = (warp - 2 - kDq) >> 2;
        const int rt = 32 * q + lane;  // weight row of the tile = TMEM lane
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + kAccCol;
        const int cbeg = 128 * e, cend = min(p.TT, cbeg + 128);  // this warp's token columns
        const bool odd = lane & 1;
        int tj = 0;
        for (int t = tile0; t < ntiles; t += tstep, ++tj) {
            const int ws = t / p.MT, ms = t % p.MT;
            if (!mbar_wait_warp(acc_full, tj & 1, p.err, 0x109)) break;
            tc_fence_after();
            if (staged) {
                // Drain the accumulator into the X stage(s) as [token][128 weight rows] (bf16:
                // all T tokens in the last stage; f32: tokens 128e.. in stage g_last - e) and
                // release it after the last TMEM load.  Each 32-token chunk leaves through a
                // TMA store as soon as the four warps of its half have staged it, so the store
                // overlaps the rest of the drain.
                const int glast = (tj + 1) * NST - 1;
                uint8_t* stg = smem + Smem::kOffX + ((glast - (out_f32 ? e : 0)) % kStages) * kXBytes;
                for (int c = cbeg; c < cend || (c == cbeg && cbeg >= cend); c += 32) {
                    uint32_t v[32];
                    const bool have = c < cend;
                    if (have) {
                        tmem_ld_32x32b_x32(tq + c, v);
                        tmem_ld_wait(v);
                    }
                    if (c + 32 >= cend) {  // everything this warp needs is in registers
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(acc_empty);
                    }
                    if (!have) break;
                    if (out_f32) {
                        float* col = reinterpret_cast<float*>(stg) + (size_t)(c - cbeg) * TW + rt;
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) col[jj * TW] = __uint_as_float(v[jj]);
                    } else {
                        uint16_t* col = reinterpret_cast<uint16_t*>(stg) + (size_t)c * TW + rt;  // token c, row rt
#pragma unroll
                        for (int jj = 0; jj < 32; jj += 2) {
                            __nv_bfloat162 b2 =
                                __floats2bfloat162_rn(__uint_as_float(v[jj]), __uint_as_float(v[jj + 1]));
                            const uint32_t bits = *reinterpret_cast<uint32_t*>(&b2);
                            col[jj * TW] = (uint16_t)(bits & 0xFFFFu);
                            col[(jj + 1) * TW] = (uint16_t)(bits >> 16);
                        }
                    }
                    if constexpr (!kGeglu) {
                        fence_proxy_async_smem();  // the generic stores, before the async-proxy read
                        if (e == 0) asm volatile("bar.sync 2, 128;" ::: "memory");  // the half's 4 warps
                        else asm volatile("bar.sync 3, 128;" ::: "memory");
                        if (q == 0 && lane == 0) {
                            const uint8_t* src = out_f32 ? stg + (size_t)(c - cbeg) * TW * 4 : stg + (size_t)c * TW * 2;
                            tma_store_2d(&ymap, src, ws * TW, plane_row0 + ms * p.TT + c);
                            bulk_commit_group();
                        }
                    }
                }
                if constexpr (kGeglu) {
                    asm volatile("bar.sync 1, %0;" ::"r"(kEpi * 32) : "memory");
                    geglu_rows(smem + Smem::kOffX + ((glast - e) % kStages) * kXBytes, q, e, lane, ms, ws, p);
                    asm volatile("bar.sync 1, %0;" ::"r"(kEpi * 32) : "memory");
                    if (warp == 2 + kDq && lane == 0)
                        for (int h = 0; h < out_stages; ++h) mbar_arrive(&load_empty[(glast - h) % kStages]);
                    continue;
                }
                if (q == 0 && lane == 0) bulk_wait_read_all();  // this half's stores have read the stage
                asm volatile("bar.sync 1, %0;" ::"r"(kEpi * 32) : "memory");
                if (warp == 2 + kDq && lane == 0)
                    for (int h = 0; h < out_stages; ++h) mbar_arrive(&load_empty[(glast - h) % kStages]);
                continue;
            }
            // Fallback (f32 output, or a partial, with fewer stages than output stages): one
            // chunk at a time, each lane stores its weight row's 32 tokens.
            const int n = ws * TW + rt;
            float* ybase = S > 1 ? p.part + (size_t)plane_row0 * p.ldy : reinterpret_cast<float*>(p.y);
            for (int c = cbeg; c < cend || (c == cbeg && cbeg >= cend); c += 32) {
                uint32_t v[32];
                const bool have = c < cend;
                if (have) {
                    tmem_ld_32x32b_x32(tq + c, v);
                    tmem_ld_wait(v);
                }
                if (c + 32 >= cend) {  // everything this warp needs is in registers
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(acc_empty);
                }
                if (!have) break;
                const int m0 = ms * p.TT + c;
                if (n < p.N) {
                    float* yp = ybase + (size_t)m0 * p.ldy + n;
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj)
                        if (m0 + jj < p.M) yp[(size_t)jj * p.ldy] = __uint_as_float(v[jj]);
                }
            }
        }
        if (staged && q == 0 && lane == 0) bulk_wait_all();  // this half's tile stores have landed
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// Split-K epilogue: y[m, n] = sum over slices s (in order) of part[s][m][n], f32 or bf16
// out; one thread per 4 columns.  Reads the planes from L2 (they were just written).
__global__ void __launch_bounds__(256) splitk_sum_kernel(const float4* __restrict__ part, int S,
                                                         long long plane4, int M, int N4, void* __restrict__ y,
                                                         int y_f32) {
    pdl_trigger();
    pdl_wait();  // the partial planes come from the GEMM
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)M * N4) return;
    float4 acc = __ldcg(part + i);
    int s = 1;
    for (; s + 4 <= S; s += 4) {  // four planes in flight, summed in slice order
        const float4 a = __ldcg(part + s * plane4 + i), b = __ldcg(part + (s + 1) * plane4 + i);
        const float4 c = __ldcg(part + (s + 2) * plane4 + i), d = __ldcg(part + (s + 3) * plane4 + i);
        acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
        acc.x += b.x; acc.y += b.y; acc.z += b.z; acc.w += b.w;
        acc.x += c.x; acc.y += c.y; acc.z += c.z; acc.w += c.w;
        acc.x += d.x; acc.y += d.y; acc.z += d.z; acc.w += d.w;
    }
    for (; s < S; ++s) {
        const float4 a = __ldcg(part + s * plane4 + i);
        acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
    }
    if (y_f32) {
        reinterpret_cast<float4*>(y)[i] = acc;
    } else {
        __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
        reinterpret_cast<uint2*>(y)[i] = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
    }
}

// GeGLU over the f32 planes of a linear whose 128-row slabs are 64 gate rows then the 64
// matching up rows: out[m, 64 s + j] = bf16(gelu(gate) * up), slices added in order.
__global__ void __launch_bounds__(256) geglu_planes_kernel(const float* __restrict__ base, int count,
                                                           long long stride, int ld, int M, int half_n,
                                                           uint16_t* __restrict__ out) {
    pdl_trigger();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)M * half_n) return;
    const int m = (int)(i / half_n), f = (int)(i - (long long)m * half_n);
    const size_t gcol = (size_t)m * ld + (f / 64) * 128 + (f % 64);
    float g = base[gcol], u = base[gcol + 64];
    for (int s = 1; s < count; ++s) {
        g += base[(size_t)s * stride + gcol];
        u += base[(size_t)s * stride + gcol + 64];
    }
    out[i] = (uint16_t)f32_to_bf16_bits(gelu_ref(g) * u);
}

}  // namespace

namespace g4 {

// Tiles: 128 weight rows x T tokens (T = M rounded up to 32, at most 256).  With at least
// one tile per SM the grid is persistent (one CTA per SM walking the tiles, token tile
// fastest so concurrent CTAs share the weight slabs in L2); otherwise K is split over S
// CTAs per tile (at most one CTA per SM in total, >= 3 weight blocks per slice) whose
// partial planes splitk_sum_kernel adds.
// planes != nullptr: leave the f32 output as partial planes in the context workspace (no
// summing pass; y is ignored) and describe them in *planes.
// geglu != nullptr (and planes == nullptr): write bf16 GeGLU activations [M, N/2] there,
// fused into the epilogue of an unsplit tile, else planes + geglu_planes_kernel.
static g4_status gemm_core(g4_ctx* ctx, const g4_linear* lin, const uint16_t* x, int M, void* y, int y_f32,
                           g4_planes* planes, uint16_t* geglu = nullptr) {
    const g4_linear_dev& L = lin->dev;
    if (!gemm_supported(lin, M)) return set_error(G4_ERR_UNSUPPORTED, "tcgen05 GEMM: shape K=%d N=%d", L.K, L.N);
    static std::atomic<uint64_t> attr_set{0};
    if (!(attr_set.load() & (1ull << ctx->device))) {
        G4_CHECK_CUDA(cudaFuncSetAttribute(gemm_w4_tmem_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           Smem::kBytes));
        G4_CHECK_CUDA(cudaFuncSetAttribute(gemm_w4_tmem_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           Smem::kBytes));
        attr_set.fetch_or(1ull << ctx->device);
    }
    if (!planes && reinterpret_cast<uintptr_t>(y) % 16 != 0)
        return set_error(G4_ERR_INVALID, "tcgen05 GEMM: y must be 16-byte aligned");
    W4Params p{};
    p.tblk = L.tblk;
    p.y = y;
    p.M = M;
    p.N = L.N;
    p.ldy = L.N;
    p.y_f32 = y_f32;
    p.Kc = L.Kc;
    p.NS = L.NS;
    p.TT = M >= TTmax ? TTmax : (M + 31) / 32 * 32;
    // A decode-size batch (128 < M <= 256) of a linear with few weight tiles: two 128-token
    // tiles instead of one 256-token tile double the CTAs without adding split-K planes and
    // halve each CTA's X load and output store, which is what such a GEMM waits on.
    // (Where the doubled tiles would not fit in one wave, the 256-token tile is faster.)
    if (M > 128 && M <= TTmax && (long long)L.NS * 2 <= ctx->num_sms) p.TT = 128;
    p.MT = (M + p.TT - 1) / p.TT;
    p.err = ctx->d_err;
    const long long ntiles = (long long)p.NS * p.MT;
    if (ntiles > 0x7fffffffLL) return set_error(G4_ERR_UNSUPPORTED, "tcgen05 GEMM: M=%d N=%d too large", M, L.N);
    int S = 1;
    // At most 8 slices: each further partial plane costs its consumer more L2 reads than
    // the extra CTAs save (decode step at M = 256).
    while (ntiles * (S + 1) <= ctx->num_sms && p.Kc / (S + 1) >= 3 && S < kMaxSlices) ++S;
    p.kper = (p.Kc + S - 1) / S;
    S = (p.Kc + p.kper - 1) / p.kper;  // no empty slice
    p.ksplit = S;
    if (geglu) {
        const int nst = (p.kper + kSub - 1) / kSub, out_stages = p.TT > 128 ? 2 : 1;
        if (S == 1 && nst >= out_stages && L.N % TW == 0) {
            p.geglu = 1;
            p.y_f32 = 1;
            y = geglu;
            p.y = y;
        } else {  // the planes, then the GeGLU pass
            g4_planes pl;
            g4_status st0 = gemm_core(ctx, lin, x, M, nullptr, 1, &pl);
            if (st0) return st0;
            const long long n = (long long)M * (L.N / 2);
            return launch(ctx, "geglu_planes_kernel", geglu_planes_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256),
                          0, 1, pl.base, pl.count, pl.stride, pl.ld, M, L.N / 2, geglu);
        }
    }
    CUtensorMap xmap, ymap;
    g4_status st = encode_tensor_map_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, const_cast<uint16_t*>(x), L.K, M,
                                        (uint64_t)L.K * 2, TK, p.TT, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    // Rows of one partial plane: whole token tiles, and whole 128-row store boxes (a box that
    // ran past the plane would write into the next slice's plane).
    const long long Mp = (long long)p.MT * (p.TT > 128 ? 256 : p.TT);
    if (planes && S == 1) {  // the whole f32 output is the one plane, in the workspace
        st = ensure_workspace(ctx, (size_t)M * L.N * 4);
        if (st) return st;
        y = ctx->ws;
        p.y = y;
        y_f32 = p.y_f32 = 1;
        *planes = g4_planes{static_cast<const float*>(ctx->ws), 1, 0, L.N};
    }
    if (S > 1) {
        // partial planes [S][Mp][N] f32 in the context workspace; boxes of [32 tokens][128 rows]
        const size_t bytes = (size_t)S * Mp * L.N * 4;
        st = ensure_workspace(ctx, bytes);
        if (st) return st;
        p.part = static_cast<float*>(ctx->ws);
        if (planes) *planes = g4_planes{p.part, S, Mp * L.N, L.N};
        st = encode_tensor_map_2d(&ymap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.part, L.N, (uint64_t)(S * Mp),
                                  (uint64_t)L.N * 4, TW, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
    } else if (p.geglu) {
        ymap = xmap;  // unused: GeGLU rows leave through plain coalesced stores
    } else {
        // Y tiles leave through TMA stores of [32 tokens][128 rows] chunks
        st = y_f32 ? encode_tensor_map_2d(&ymap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, y, L.N, M, (uint64_t)L.N * 4, TW, 32,
                                          CU_TENSOR_MAP_SWIZZLE_NONE)
                   : encode_tensor_map_2d(&ymap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, y, L.N, M, (uint64_t)L.N * 2, TW, 32,
                                          CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    if (st) return st;
    const unsigned grid = S > 1 ? (unsigned)(ntiles * S) : (unsigned)std::min<long long>(ntiles, ctx->num_sms);
    p.wsplit = (S > 1 || ntiles <= ctx->num_sms) ? 1 : 0;  // every CTA one tile (or one K slice of one)
    st = p.geglu ? launch(ctx, "gemm_w4_tmem_kernel<geglu>", gemm_w4_tmem_kernel<true>, dim3(grid), dim3(kThreads),
                          Smem::kBytes, 1, xmap, ymap, p)
                 : launch(ctx, "gemm_w4_tmem_kernel", gemm_w4_tmem_kernel<false>, dim3(grid), dim3(kThreads),
                          Smem::kBytes, 1, xmap, ymap, p);
    if (st || S == 1 || planes) return st;
    const long long n4 = (long long)M * (L.N / 4);
    return launch(ctx, "splitk_sum_kernel", splitk_sum_kernel, dim3((unsigned)((n4 + 255) / 256)), dim3(256), 0, 1,
                  reinterpret_cast<const float4*>(p.part), S, Mp * (L.N / 4), M, L.N / 4, y, y_f32);
}

g4_status launch_gemm(g4_ctx* ctx, const g4_linear* lin, const uint16_t* x, int M, void* y, int y_f32) {
    return gemm_core(ctx, lin, x, M, y, y_f32, nullptr);
}

g4_status launch_gemm_planes(g4_ctx* ctx, const g4_linear* lin, const uint16_t* x, int M, g4_planes* planes) {
    return gemm_core(ctx, lin, x, M, nullptr, 1, planes);
}

g4_status launch_gemm_geglu(g4_ctx* ctx, const g4_linear* lin, const uint16_t* x, int M, uint16_t* out) {
    return gemm_core(ctx, lin, x, M, nullptr, 1, nullptr, out);
}

g4_status launch_geglu_planes(g4_ctx* ctx, const g4_planes& pl, int M, int N, uint16_t* out) {
    const long long n = (long long)M * (N / 2);
    return launch(ctx, "geglu_planes_kernel", geglu_planes_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, 1,
                  pl.base, pl.count, pl.stride, pl.ld, M, N / 2, out);
}

}  // namespace g4
