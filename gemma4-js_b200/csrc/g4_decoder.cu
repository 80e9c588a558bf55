// g4_decoder.cu -- one greedy decode step of one sequence in one persistent launch.
//
// The reference decodes a token as a chain of ~420 dependent operator dispatches
// (encodeLayer, custom-webgpu/gemma4-webgpu.js:215-310; forward :311-412; greedy :441-480),
// and the op-by-op path of this library mirrors it as ~430 kernel launches, each paying a
// launch and an L2 round trip on a few MB of weights.  Here one kernel, one CTA per SM (a
// cooperative launch, so all CTAs are resident), runs the whole token as phases separated by
// grid-wide barriers (8 per layer):
//
//   embed + top proj + q/k/v | attention tiles | combine | o | gate/up+GeGLU | down |
//   PLE gate | PLE proj | ... x 35 layers ... | LM head + softcap + argmax | pick
//
// Every W4A16 linear is split into units (16 weight rows x a K slice, or a gate/up pair of
// 16-row tiles); each CTA owns a contiguous range of units and, one linear ahead, pulls their
// int4 blocks and scales into shared memory with bulk copies (two buffers: while linear w is
// computed from one, linear w+1 streams into the other), so the weights stream while the
// barriers resolve.  Row-wise operators (RMS norms, residual, GeGLU, PLE mix) are computed
// redundantly by every CTA from the f32 partial results in L2, which keeps the residual stream
// in each CTA's shared memory and saves a barrier per operator; each CTA reads in its own
// rotated order so that 148 CTAs do not queue on the same L2 lines.  The attention combine is
// split over the CTAs.  On this GPU a dependent L2 round trip costs about a microsecond, so
// every such operator issues all of its loads before it uses any.  The phase and layer descriptors are
// copied into shared memory once per step (an acquire at each barrier drops L1 contents).
// The arithmetic is the op path's: exact int4 x bf16 products on mma.m16n8k16 with FP32
// accumulation, bf16 activations into every linear, f32 norms, bf16 K/V/q.
//
// Barrier: each CTA adds one to an arrival counter (acquire-release); the CTA that completes
// it resets the counter and releases a generation word, which the others poll (on its own
// line).  The generation only grows: each CTA reads it on entry, before any CTA can complete
// the first barrier, and waits for it to move past that value barrier by barrier.  Every wait
// is bounded in wall time; a CTA that gives up raises G4_DEVERR_TIMEOUT and sets an abort word
// that every other wait polls, so the grid winds down instead of hanging (g4_decoder_reset
// clears the words).
#include <stdio.h>

#include <algorithm>
#include <vector>

#include "g4_attention.cuh"
#include "g4_common.cuh"
#include "g4_dense.cuh"
#include "g4_linear.cuh"
#include "g4_ple.cuh"

namespace {

using namespace g4dev;

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kBlockW = 512;    // bytes of int4 weights per 16-row x 64-column block
constexpr int kBlockS = 64;     // bytes of scales per block
constexpr int kMaxTiles = 256;  // key tiles of one attention (16384 / hd keys each)
constexpr int kMaxSmem = 232448;
constexpr int kMaxH = 2048;
constexpr int kMaxSplits = 8;
constexpr int kBars = 5;        // mbarriers: weight buffers 0/1, attention, head stages 1/3

enum : int { kPlanes = 0, kGeglu = 1 };

struct WPhase {
    const uint4* wfrag;
    const uint2* sfrag;
    int K, N, Kc, NT;
    int kind;   // kPlanes: unit u = (nt = u / S, split = u % S), bpu blocks; kGeglu: unit = gate/up tile pair
    int S, bpu, units;
    float* planes;      // kPlanes: [S][N] f32 partial sums, added in split order by the consumer
    uint16_t* act;      // kGeglu: [N / 2] bf16 = gelu(gate) * up
};

struct DLayer {
    int wq, wo, wgu, wd, wpg, wpp;  // weight-phase indices
    const float *n_pa, *n_pf, *n_pff, *n_pple, *qn, *kn, *w_next;
    float skip;
    uint16_t *kc, *vc;  // bf16 caches [capacity, hd]; row = position
    int hd, full, has_kv, rope_angles, inter;
    float rope_base;
};
static_assert(sizeof(WPhase) % 16 == 0 && sizeof(DLayer) % 16 == 0, "descriptors are copied as uint4");

struct DParams {
    int L, H, heads, pdim, vocab, window, cap, nph;
    float eps, softcap, proj_scale;  // proj_scale = 1 / sqrt(H)
    const uint16_t* embed;  // [vocab, H] bf16: the embedding and the tied head
    const uint8_t* ple_packed;
    const uint16_t* ple_scales;
    int ple_width;
    const float *ple_norm, *n_in0;
    const WPhase* ph;
    const DLayer* layers;
    float* attn_part;     // [kMaxTiles][heads][hd + 2]
    uint16_t* attn_out;   // [heads * hd] bf16: the combined attention, input of the o projection
    float2* head_part;    // [gridDim.x] (capped value, index)
    unsigned* sync;       // barrier words, each on its own 128-byte line (kSync*)
    unsigned long long* timeline;  // optional: globaltimer stamps, timeline_cap per CTA
    int timeline_cap;
    uint32_t* err;
    const int32_t* ids;
    int32_t* seq_pos;
    int32_t* next;
    float* val;
    // shared-memory plan (byte offsets)
    int off_h, off_x, off_q, off_p, off_red, off_sred, off_bar, off_ph, off_ly, off_rope, off_w0, wbuf;
    int head_rows;  // vocabulary rows per head stage (half a weight buffer)
    // RoPE of the two layer kinds (0 sliding, 1 global): hd, base, rotated pairs
    int rope_hd[2], rope_n[2];
    float rope_base[2];
};

constexpr int kSyncCount = 0, kSyncGen = 32, kSyncAbort = 64;  // words, each on its own 128-byte line
constexpr int kSyncBytes = 96 * 4;

// ------------------------------------------------------------------ grid barrier ----

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned atom_add_acqrel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void st_relaxed(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct Grid {
    unsigned* sync;
    uint32_t* err;
    unsigned n;     // CTAs
    unsigned gen;   // generation seen (thread 0)
    unsigned long long* tl;  // this CTA's timeline row (thread 0, may be null)
    int tl_cap, tl_n;
    __device__ __forceinline__ void mark() {
        if (tl && tl_n < tl_cap) tl[tl_n++] = globaltimer_ns();
    }
};

// All CTAs meet; false when the grid is aborting (this CTA then winds down).  Each CTA adds one
// to the arrival counter (acquire-release: it publishes this CTA's writes, which bar.sync
// ordered before it); the CTA that completes the count resets it and releases the generation
// word the others poll.  Two dependent L2 round trips on the critical path.
__device__ bool grid_sync(Grid& gr, int* s_flag, uint32_t site) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        gr.mark();
        if (atom_add_acqrel(gr.sync + kSyncCount, 1u) == gr.n - 1) {
            st_relaxed(gr.sync + kSyncCount, 0u);
            red_release_add(gr.sync + kSyncGen, 1u);  // ordered after the reset
        } else {
            const unsigned long long t0 = globaltimer_ns();
            unsigned spins = 0;
            while (ld_acquire_u32(gr.sync + kSyncGen) == gr.gen) {
                if ((++spins & 63u) == 0) {
                    if (ld_acquire_u32(gr.sync + kSyncAbort)) {
                        ok = 0;
                        break;
                    }
                    if (globaltimer_ns() - t0 > kWaitLimitNs) {
                        raise_error(gr.err, G4_DEVERR_TIMEOUT, site);
                        atomicExch(gr.sync + kSyncAbort, 1u);
                        ok = 0;
                        break;
                    }
                }
            }
        }
        gr.gen += 1;
        gr.mark();
        *s_flag = ok;
    }
    __syncthreads();
    return *s_flag != 0;
}

// ------------------------------------------------------------------ block helpers ----

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// Sum over the CTA (every thread gets it); sred holds kWarps floats.
__device__ __forceinline__ float block_sum(float v, float* sred) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sred[w] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) s += sred[i];
    return s;
}

__device__ __forceinline__ float bf16r(float v) { return bf16_bits_to_f32(f32_to_bf16_bits(v)); }
__device__ __forceinline__ float lo_bf16(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf16(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// ------------------------------------------------------------- weight prefetch ----

__device__ __forceinline__ void unit_range(const WPhase& ph, int& u0, int& u1) {
    u0 = (int)((long long)ph.units * blockIdx.x / gridDim.x);
    u1 = (int)((long long)ph.units * (blockIdx.x + 1) / gridDim.x);
}
// Blocks of unit u (per tile) and its first K block.
__device__ __forceinline__ void unit_blocks(const WPhase& ph, int u, int& nt0, int& nt1, int& c0, int& nb) {
    if (ph.kind == kGeglu) {
        const int s = u >> 2, i = u & 3;
        nt0 = 8 * s + i;
        nt1 = 8 * s + 4 + i;
        c0 = 0;
        nb = ph.Kc;
    } else {
        nt0 = nt1 = u / ph.S;
        c0 = (u % ph.S) * ph.bpu;
        nb = min(ph.bpu, ph.Kc - c0);
    }
}
// Bytes of this CTA's units (weights then scales).
__device__ int phase_bytes(const WPhase& ph, int u0, int u1, int* wbytes) {
    int blocks = 0;
    for (int u = u0; u < u1; ++u) {
        int a, b, c0, nb;
        unit_blocks(ph, u, a, b, c0, nb);
        blocks += nb * (ph.kind == kGeglu ? 2 : 1);
    }
    *wbytes = blocks * kBlockW;
    return blocks * (kBlockW + kBlockS);
}
// Thread 0: one mbarrier transaction for all weight and scale blocks of this CTA's units,
// laid out [unit][tile][block] x 512 B, then the scales in the same order x 64 B.
__device__ bool issue_phase(const WPhase& ph, uint8_t* buf, uint64_t* bar) {
    int u0, u1, wbytes;
    unit_range(ph, u0, u1);
    if (u0 >= u1) return false;
    if (threadIdx.x == 0) {
        const int total = phase_bytes(ph, u0, u1, &wbytes);
        fence_proxy_async_smem();  // earlier generic accesses of this buffer come first
        mbar_arrive_expect_tx(bar, (uint32_t)total);
        int wo = 0, so = wbytes;
        for (int u = u0; u < u1; ++u) {
            int nt[2], c0, nb;
            unit_blocks(ph, u, nt[0], nt[1], c0, nb);
            const int tiles = ph.kind == kGeglu ? 2 : 1;
            for (int tl = 0; tl < tiles; ++tl) {
                const size_t blk = (size_t)nt[tl] * ph.Kc + c0;
                bulk_load(buf + wo, ph.wfrag + blk * 32, nb * kBlockW, bar);
                bulk_load(buf + so, ph.sfrag + blk * 8, nb * kBlockS, bar);
                wo += nb * kBlockW;
                so += nb * kBlockS;
            }
        }
    }
    return true;
}

// ------------------------------------------------------------------- GEMV math ----

// acc += the 16 rows x 64 columns block (weights wblk, scales sblk) times x[c*64 .. +64]
// for token 0 (lanes with g == 0 carry the activation; the other 7 columns are zero).
__device__ __forceinline__ void gemv_block(float (&acc)[4], const uint8_t* wblk, const uint8_t* sblk,
                                           const uint16_t* x, int c, int lane) {
    const int g = lane >> 2, t = lane & 3;
    const uint4 wv = *reinterpret_cast<const uint4*>(wblk + lane * 16);
    const uint2 sv = *reinterpret_cast<const uint2*>(sblk + g * 8);
    const uint32_t wq[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int G = 0; G < 2; ++G) {
        const uint32_t w0 = wq[2 * G], w1 = wq[2 * G + 1];
        const uint32_t a0[4] = {int4pair_to_bf16x2(w0), int4pair_to_bf16x2(w1), int4pair_to_bf16x2(w0 >> 4),
                                int4pair_to_bf16x2(w1 >> 4)};
        const uint32_t a1[4] = {int4pair_to_bf16x2(w0 >> 8), int4pair_to_bf16x2(w1 >> 8),
                                int4pair_to_bf16x2(w0 >> 12), int4pair_to_bf16x2(w1 >> 12)};
        const uint32_t sw = G ? sv.y : sv.x;
        const float s_lo = bf16_bits_to_f32(sw & 0xFFFFu), s_hi = bf16_bits_to_f32(sw >> 16);
        uint4 xg = make_uint4(0, 0, 0, 0);
        if (g == 0) xg = *reinterpret_cast<const uint4*>(x + c * 64 + G * 32 + t * 8);
        const uint32_t b0[2] = {xg.x, xg.y}, b1[2] = {xg.z, xg.w};
        float d[4];
        const float z[4] = {0.f, 0.f, 0.f, 0.f};
        mma_bf16_16816(d, a0, b0, z);
        mma_bf16_16816(d, a1, b1, d);
        acc[0] = fmaf(s_lo, d[0], acc[0]);
        acc[2] = fmaf(s_hi, d[2], acc[2]);
    }
}

// The linear of weight phase `ph` on x (bf16 in shared memory) from the staged blocks in buf.
// Partial planes: plane[split][row]; GeGLU: act[col] = bf16(gelu(gate) * up).
__device__ void gemv_phase(const WPhase& ph, const uint8_t* buf, const uint16_t* x, float* red) {
    int u0, u1, wbytes;
    unit_range(ph, u0, u1);
    if (u0 >= u1) return;
    phase_bytes(ph, u0, u1, &wbytes);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int tiles = ph.kind == kGeglu ? 2 : 1;
    int boff = 0;  // block offset of the unit in the buffer
    for (int u = u0; u < u1; ++u) {
        int nt[2], c0, nb;
        unit_blocks(ph, u, nt[0], nt[1], c0, nb);
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        for (int tl = 0; tl < tiles; ++tl) {
            const int tb = boff + tl * nb;
            for (int b = warp; b < nb; b += kWarps)
                gemv_block(acc[tl], buf + (size_t)(tb + b) * kBlockW, buf + wbytes + (size_t)(tb + b) * kBlockS, x,
                           c0 + b, lane);
        }
        // reduce the warps: red[warp][tile][2][32]
#pragma unroll
        for (int tl = 0; tl < 2; ++tl) {
            red[((warp * 2 + tl) * 2 + 0) * 32 + lane] = acc[tl][0];
            red[((warp * 2 + tl) * 2 + 1) * 32 + lane] = acc[tl][2];
        }
        __syncthreads();
        if (warp == 0 && t == 0) {
            float v[2][2];
#pragma unroll
            for (int tl = 0; tl < 2; ++tl)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float s = 0.f;
#pragma unroll
                    for (int w = 0; w < kWarps; ++w) s += red[((w * 2 + tl) * 2 + h) * 32 + lane];
                    v[tl][h] = s;
                }
            if (ph.kind == kGeglu) {
                const int s = u >> 2, i = u & 3;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int col = 64 * s + 16 * i + g + 8 * h;
                    if (col < ph.N / 2) ph.act[col] = (uint16_t)f32_to_bf16_bits(gelu_ref(v[0][h]) * v[1][h]);
                }
            } else {
                const int split = u % ph.S;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int row = nt[0] * 16 + g + 8 * h;
                    if (row < ph.N) ph.planes[(size_t)split * ph.N + row] = v[0][h];
                }
            }
        }
        __syncthreads();
        boff += nb * tiles;
    }
}

// Sum of the S <= 8 planes of element i (in split order), from L2 (written by other CTAs):
// all loads are issued before the adds, one L2 round trip instead of S.
__device__ __forceinline__ float plane_sum(const WPhase& ph, int i) {
    float v[kMaxSplits];
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s) v[s] = s < ph.S ? __ldcg(ph.planes + (size_t)s * ph.N + i) : 0.f;
    float a = v[0];
#pragma unroll
    for (int s = 1; s < kMaxSplits; ++s)
        if (s < ph.S) a += v[s];
    return a;
}

// Every CTA reads the same few KB at the same moment in the row-wise operators; a CTA-rotated
// element order spreads those concurrent requests over the L2 slices (rot: a 128-byte line
// step per CTA).  Values are staged in shared memory and the arithmetic then runs in one fixed
// order, so every CTA computes the same bits.
__device__ __forceinline__ int rot_of(int n) { return (int)((blockIdx.x * 32u) % (unsigned)n); }

// Residual update and the next linear's input (post_norm_add_kernel's arithmetic):
//   h = (h + rms(y) * w_post) * skip;  x = bf16(w_next ? rms(h) * w_next : h)
// stage: >= 3 H floats of an idle buffer (y, w_post, w_next).  One L2 round trip.
__device__ void post_norm_add(const WPhase& ph, float* h, const float* w_post, float skip, const float* w_next,
                              int H, float eps, uint16_t* x, float* sred, float* stage) {
    constexpr int kPer = kMaxH / kThreads;
    float* ys = stage;
    float* wps = stage + H;
    float* wns = stage + 2 * H;
    const int rot = rot_of(H);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {  // every load first, in this CTA's rotated order
        int i = threadIdx.x + j * kThreads;
        if (i < H) {
            i += rot;
            if (i >= H) i -= H;
            const float y = plane_sum(ph, i);
            const float a = __ldg(w_post + i);
            const float b = w_next ? __ldg(w_next + i) : 0.f;
            ys[i] = y;
            wps[i] = a;
            wns[i] = b;
        }
    }
    __syncthreads();
    float y[kPer];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int i = threadIdx.x + j * kThreads;
        y[j] = i < H ? ys[i] : 0.f;
        ss += y[j] * y[j];
    }
    const float inv = rsqrtf(block_sum(ss, sred) / (float)H + eps);
    float ss2 = 0.f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int i = threadIdx.x + j * kThreads;
        if (i < H) {
            const float hn = (h[i] + y[j] * inv * wps[i]) * skip;
            h[i] = hn;
            y[j] = hn;
            ss2 += hn * hn;
        }
    }
    const float inv2 = w_next ? rsqrtf(block_sum(ss2, sred) / (float)H + eps) : 1.f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int i = threadIdx.x + j * kThreads;
        if (i < H) x[i] = (uint16_t)f32_to_bf16_bits(w_next ? y[j] * inv2 * wns[i] : y[j]);
    }
    __syncthreads();
}

// x = bf16 rows written by other CTAs (attention output, GeGLU activation), rotated per CTA.
__device__ void load_x(uint16_t* x, const uint16_t* src, int n) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(x);
    const int n8 = n / 8, rot = (int)((blockIdx.x * 8u) % (unsigned)n8);
    for (int i = threadIdx.x; i < n8; i += kThreads) {
        int k = i + rot;
        if (k >= n8) k -= n8;
        d[k] = __ldcg(s + k);
    }
    __syncthreads();
}

// ------------------------------------------------------------------- attention ----

// cos/sin of theta_i = pos / base^(2i/hd) for the pairs of both layer kinds (NORM_ROPE_SHADER
// :1197-1198), once per step: rope[kind * 512 + i] = cos, rope[kind * 512 + 256 + i] = sin.
__device__ void rope_tables(const DParams& P, int pos, float* rope) {
    for (int k = 0; k < 2; ++k)
        for (int i = threadIdx.x; i < 256; i += kThreads) {
            float cs = 1.f, sn = 0.f;
            if (i < P.rope_n[k]) {
                const float theta = (float)pos / powf(P.rope_base[k], 2.f * (float)i / (float)P.rope_hd[k]);
                sn = sinf(theta);
                cs = cosf(theta);
            }
            rope[k * 512 + i] = cs;
            rope[k * 512 + 256 + i] = sn;
        }
}

// q (all heads) and, for slot heads / heads + 1, k / v of the current position, from the
// qkv planes: RMS over the head, q/k norm scale, RoPE (NORM_ROPE_SHADER), bf16-rounded.
// Warp w handles slots w, w + 8, ...; lane owns the rotation pairs (i, i + HD/2), i = lane + 32j.
template <int HD>
__device__ void qkv_slots(const WPhase& ph, const DLayer& ly, int heads, float eps, int s0, int s1,
                          const float* rope, float* q, float* kv_out) {
    constexpr int HALF = HD / 2, NP = HALF / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int slot = s0 + warp; slot < s1; slot += kWarps) {
        const float* sc = slot < heads ? ly.qn : (slot == heads ? ly.kn : nullptr);
        float a0[NP], a1[NP], c0[NP], c1[NP];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < NP; ++j) {  // all loads of the slot in flight together
            const int i = lane + 32 * j;
            a0[j] = plane_sum(ph, slot * HD + i);
            a1[j] = plane_sum(ph, slot * HD + i + HALF);
            c0[j] = sc ? __ldg(sc + i) : 1.f;
            c1[j] = sc ? __ldg(sc + i + HALF) : 1.f;
        }
#pragma unroll
        for (int j = 0; j < NP; ++j) ss += a0[j] * a0[j] + a1[j] * a1[j];
        const float inv = rsqrtf(warp_sum(ss) / (float)HD + eps);
        float* dst = slot < heads ? q + slot * HD : kv_out + (slot - heads) * HD;
#pragma unroll
        for (int j = 0; j < NP; ++j) {
            const int i = lane + 32 * j;
            const float x0 = a0[j] * inv * c0[j], x1 = a1[j] * inv * c1[j];
            if (!sc) {  // v: RMS without scale
                dst[i] = bf16r(x0);
                dst[i + HALF] = bf16r(x1);
                continue;
            }
            const float cs = rope[i], sn = rope[256 + i];  // this layer kind's table
            dst[i] = bf16r(x0 * cs - x1 * sn);
            dst[i + HALF] = bf16r(x1 * cs + x0 * sn);
        }
    }
    __syncthreads();
}

// One tile of keys [k0, k1) (all valid for the single query at `pos`): logits, partial
// softmax and P.V for every head, written as (m, l, o[HD]) to part[head].
// Logits: warp per key; lane owns dims lane*4 + 128c; each lane's 8 per-head partial dots
// are reduced across the warp in one transposed butterfly (9 shuffles for all 8 heads).
// pT holds the probabilities as [key][8 heads].
template <int HD>
__device__ void attend_tile(const uint16_t* Kt, const uint16_t* Vt, int n, int heads, const float* q, float* pT,
                            float* part) {
    constexpr int C = HD / 128;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int j = warp; j < n; j += kWarps) {
        float kf[4 * C];
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const uint2 kv = *reinterpret_cast<const uint2*>(Kt + (size_t)j * HD + c * 128 + lane * 4);
            kf[4 * c + 0] = lo_bf16(kv.x);
            kf[4 * c + 1] = hi_bf16(kv.x);
            kf[4 * c + 2] = lo_bf16(kv.y);
            kf[4 * c + 3] = hi_bf16(kv.y);
        }
        float v[8];
#pragma unroll
        for (int h = 0; h < 8; ++h) {
            float s = 0.f;
            if (h < heads) {
#pragma unroll
                for (int c = 0; c < C; ++c) {
                    const float4 qv = *reinterpret_cast<const float4*>(q + h * HD + c * 128 + lane * 4);
                    s = fmaf(qv.x, kf[4 * c + 0], s);
                    s = fmaf(qv.y, kf[4 * c + 1], s);
                    s = fmaf(qv.z, kf[4 * c + 2], s);
                    s = fmaf(qv.w, kf[4 * c + 3], s);
                }
            }
            v[h] = s;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // lanes with bit 4 keep heads 4..7, the others 0..3
            const bool up = lane & 16;
            const float got = __shfl_xor_sync(0xffffffffu, up ? v[i] : v[i + 4], 16);
            v[i] = (up ? v[i + 4] : v[i]) + got;
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {  // bit 3: + 2
            const bool up = lane & 8;
            const float got = __shfl_xor_sync(0xffffffffu, up ? v[i] : v[i + 2], 8);
            v[i] = (up ? v[i + 2] : v[i]) + got;
        }
        {  // bit 2: + 1
            const bool up = lane & 4;
            const float got = __shfl_xor_sync(0xffffffffu, up ? v[0] : v[1], 4);
            v[0] = (up ? v[1] : v[0]) + got;
        }
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
        const int hsel = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
        if ((lane & 3) == 0 && hsel < heads) pT[j * 8 + hsel] = v[0];
    }
    __syncthreads();
    // softmax partial per head: warp h
    for (int h = warp; h < heads; h += kWarps) {
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, pT[j * 8 + h]);
        m = warp_max(m);
        float l = 0.f;
        for (int j = lane; j < n; j += 32) {
            const float p = expf(pT[j * 8 + h] - m);
            pT[j * 8 + h] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) {
            part[(size_t)h * (HD + 2) + HD] = m;
            part[(size_t)h * (HD + 2) + HD + 1] = l;
        }
    }
    __syncthreads();
    // P.V: thread owns columns d = tid (+ 256); the 8 probabilities of a key are two float4
#pragma unroll
    for (int dd = 0; dd < HD / kThreads; ++dd) {
        const int d = threadIdx.x + dd * kThreads;
        float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int j = 0; j < n; ++j) {
            const float vv = bf16_bits_to_f32(Vt[(size_t)j * HD + d]);
            const float4 p0 = *reinterpret_cast<const float4*>(pT + j * 8);
            const float4 p1 = *reinterpret_cast<const float4*>(pT + j * 8 + 4);
            o[0] = fmaf(p0.x, vv, o[0]);
            o[1] = fmaf(p0.y, vv, o[1]);
            o[2] = fmaf(p0.z, vv, o[2]);
            o[3] = fmaf(p0.w, vv, o[3]);
            o[4] = fmaf(p1.x, vv, o[4]);
            o[5] = fmaf(p1.y, vv, o[5]);
            o[6] = fmaf(p1.z, vv, o[6]);
            o[7] = fmaf(p1.w, vv, o[7]);
        }
#pragma unroll
        for (int h = 0; h < 8; ++h)
            if (h < heads) part[(size_t)h * (HD + 2) + d] = o[h];
    }
}

// The tiles' partials combined, CTA c taking outputs [E c / G, E (c + 1) / G) of the E = heads
// x HD values: out[h][d] = bf16(sum_t w_t o_t[h][d] / sum_t w_t l_t[h]), w_t = exp(m_t[h] - M[h]).
// Thread (k, chunk) holds output k's tiles chunk, chunk + nchunk, ... (kPer of them per round;
// one round unless the context is very long); the first round's loads and all (m, l) pairs are
// issued before any is used.  ml: [ntile][heads] (m -> weight, l); acc: [kThreads]; den: [heads].
template <int HD>
__device__ void combine_tiles(const float* parts, int ntile, int heads, float* ml, float* acc, float* den,
                              uint16_t* out) {
    constexpr int kPer = 16;
    const size_t tstride = (size_t)heads * (HD + 2);
    const int E = heads * HD;
    const int e0 = (int)((long long)E * blockIdx.x / gridDim.x), e1 = (int)((long long)E * (blockIdx.x + 1) / gridDim.x);
    const int nout = e1 - e0;
    const int nchunk = nout > 0 ? max(1, kThreads / nout) : 1;
    const int k = threadIdx.x / nchunk, chunk = threadIdx.x - k * nchunk;
    const bool active = k < nout;
    const int e = e0 + k, hh = active ? e / HD : 0, d = e - hh * HD;
    const float* pd = parts + (size_t)hh * (HD + 2) + d;
    float v[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int t = chunk + j * nchunk;
        v[j] = (active && t < ntile) ? __ldcg(pd + (size_t)t * tstride) : 0.f;
    }
    for (int i = threadIdx.x; i < ntile * heads; i += kThreads) {
        const float* pe = parts + (size_t)(i / heads) * tstride + (size_t)(i % heads) * (HD + 2);
        ml[2 * i] = __ldcg(pe + HD);
        ml[2 * i + 1] = __ldcg(pe + HD + 1);
    }
    __syncthreads();
    if ((int)threadIdx.x < heads) {
        const int h = threadIdx.x;
        float mx = -INFINITY;
        for (int t = 0; t < ntile; ++t) mx = fmaxf(mx, ml[2 * (t * heads + h)]);
        float dn = 0.f;
        for (int t = 0; t < ntile; ++t) {
            const int i = t * heads + h;
            const float wv = expf(ml[2 * i] - mx);
            ml[2 * i] = wv;
            dn += wv * ml[2 * i + 1];
        }
        den[h] = dn;
    }
    __syncthreads();
    float o = 0.f;
    for (int base = 0;; base += kPer * nchunk) {
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int t = base + chunk + j * nchunk;
            if (active && t < ntile) o = fmaf(ml[2 * (t * heads + hh)], v[j], o);
        }
        if (base + kPer * nchunk >= ntile) break;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {  // the next round's loads (long contexts only)
            const int t = base + kPer * nchunk + chunk + j * nchunk;
            v[j] = (active && t < ntile) ? __ldcg(pd + (size_t)t * tstride) : 0.f;
        }
    }
    acc[threadIdx.x] = o;
    __syncthreads();
    if (active && chunk == 0) {
        float sum = 0.f;
        for (int c = 0; c < nchunk; ++c) sum += acc[k * nchunk + c];  // chunks in order
        out[e] = (uint16_t)f32_to_bf16_bits(sum / den[hh]);
    }
    __syncthreads();
}

// ------------------------------------------------------------------------ kernel ----

__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(DParams P) {
    extern __shared__ __align__(128) uint8_t sm[];
    float* h_s = reinterpret_cast<float*>(sm + P.off_h);
    uint16_t* x_s = reinterpret_cast<uint16_t*>(sm + P.off_x);
    float* q_s = reinterpret_cast<float*>(sm + P.off_q);
    float* p_s = reinterpret_cast<float*>(sm + P.off_p);
    float* red = reinterpret_cast<float*>(sm + P.off_red);
    float* sred = reinterpret_cast<float*>(sm + P.off_sred);
    int* s_flag = reinterpret_cast<int*>(sred + 32);
    uint64_t* wbar = reinterpret_cast<uint64_t*>(sm + P.off_bar);  // kBars mbarriers
    WPhase* sph = reinterpret_cast<WPhase*>(sm + P.off_ph);
    DLayer* sly = reinterpret_cast<DLayer*>(sm + P.off_ly);
    float* rope_s = reinterpret_cast<float*>(sm + P.off_rope);  // [2][cos, sin][256]
    uint8_t* wbuf[2] = {sm + P.off_w0, sm + P.off_w0 + P.wbuf};

    if (ld_acquire_u32(P.sync + kSyncAbort)) return;  // a previous launch aborted: wait for g4_decoder_reset
    Grid gr{P.sync, P.err, gridDim.x, 0u, nullptr, 0, 0};
    if (threadIdx.x == 0) gr.gen = ld_acquire_u32(P.sync + kSyncGen);  // before this CTA's first arrival
    if (threadIdx.x == 0 && P.timeline) {
        gr.tl = P.timeline + (size_t)blockIdx.x * P.timeline_cap;
        gr.tl_cap = P.timeline_cap;
        gr.mark();
    }
    const int nph = P.nph;
    uint32_t par[kBars] = {0, 0, 0, 0, 0};
    bool pend[kBars] = {false, false, false, false, false};

    if (threadIdx.x == 0) {
        for (int i = 0; i < kBars; ++i) mbar_init(&wbar[i], 1);
        fence_mbar_init();
    }
    // the plan (phase and layer descriptors) into shared memory: read once, not after every barrier
    {
        const uint4* src = reinterpret_cast<const uint4*>(P.ph);
        uint4* dst = reinterpret_cast<uint4*>(sph);
        for (int i = threadIdx.x; i < nph * (int)(sizeof(WPhase) / 16); i += kThreads) dst[i] = src[i];
        src = reinterpret_cast<const uint4*>(P.layers);
        dst = reinterpret_cast<uint4*>(sly);
        for (int i = threadIdx.x; i < P.L * (int)(sizeof(DLayer) / 16); i += kThreads) dst[i] = src[i];
    }
    __syncthreads();

    const int H = P.H;
    const int id_raw = P.ids[0];
    const int pos = P.seq_pos[0];
    const bool id_ok = (unsigned)id_raw < (unsigned)P.vocab;
    const int id = id_ok ? id_raw : 0;
    if (!id_ok && blockIdx.x == 0 && threadIdx.x == 0) raise_error(P.err, G4_DEVERR_BAD_INDEX);
    if (pos < 0 || pos >= P.cap) {  // every CTA sees the same position: all leave here
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            raise_error(P.err, G4_DEVERR_BAD_INDEX);
            P.next[0] = 0;
        }
        return;
    }
    const int L = pos + 1;  // keys of the query
    bool ok = true;

    // A copy wait that gives up also stops the other CTAs at their next barrier.
    auto copy_wait = [&](int b, uint32_t site) -> bool {
        const bool got = mbar_wait(&wbar[b], par[b], P.err, site);
        par[b] ^= 1u;
        pend[b] = false;
        if (!got) atomicExch(P.sync + kSyncAbort, 1u);
        return got;
    };
    auto mark = [&]() {
        if (threadIdx.x == 0) gr.mark();
    };

    // the first linear (top projection) streams in while the embedding row is read
    pend[0] = issue_phase(sph[0], wbuf[0], &wbar[0]);

    rope_tables(P, pos, rope_s);
    // embedding (gemma4-webgpu.js:199, :318): h = row * sqrt(H); the top projection reads bf16(h)
    const float esc = sqrtf((float)H);
    for (int i = threadIdx.x; i < H; i += kThreads) {
        const float v = id_ok ? bf16_bits_to_f32(P.embed[(size_t)id * H + i]) * esc : 0.f;
        h_s[i] = v;
        x_s[i] = (uint16_t)f32_to_bf16_bits(v);
    }
    __syncthreads();

    // Weight phase w computes from wbuf[w & 1].  Phase w + 1 is requested into the other buffer
    // when w starts: that buffer held w - 1 (done), and between the q/k/v phase and the o phase
    // it is the q/k/v buffer that is idle, which the attention tiles and the combine then use.
    int wcur = 0;
    auto compute_weights = [&](int w) -> bool {
        const int b = w & 1;
        if (w + 1 < nph) pend[b ^ 1] = issue_phase(sph[w + 1], wbuf[b ^ 1], &wbar[b ^ 1]);
        if (pend[b] && !copy_wait(b, 0x51)) return false;
        mark();  // weights in shared memory
        gemv_phase(sph[w], wbuf[b], x_s, red);
        __syncthreads();
        mark();  // linear done
        return true;
    };

    // top projection (per_layer_model_projection) on bf16(h), then x = bf16(rms(h) * n_in[0])
    ok = compute_weights(wcur++);
    if (ok) {
        float ss = 0.f;
        for (int i = threadIdx.x; i < H; i += kThreads) ss += h_s[i] * h_s[i];
        const float inv = rsqrtf(block_sum(ss, sred) / (float)H + P.eps);
        for (int i = threadIdx.x; i < H; i += kThreads)
            x_s[i] = (uint16_t)f32_to_bf16_bits(h_s[i] * inv * P.n_in0[i]);
        __syncthreads();
    }

    const WPhase& top = sph[0];
    for (int l = 0; l < P.L && ok; ++l) {
        const DLayer& ly = sly[l];
        const int hd = ly.hd, KT = 16384 / hd;
        // ---- q/k/v ----
        if (!(ok = compute_weights(wcur++))) break;
        if (!(ok = grid_sync(gr, s_flag, 0x52))) break;
        // ---- attention over the key tiles: CTA c owns tiles c, c + G, ... ----
        const int kstart = ly.full ? 0 : max(0, L - P.window);
        const int ntile = (L - kstart + KT - 1) / KT;
        const WPhase& pq = sph[ly.wq];
        bool have_q = false;
        uint8_t* abuf = wbuf[ly.wq & 1];  // the q/k/v buffer is free until the gate/up prefetch
        for (int tile = blockIdx.x; tile < ntile && ok; tile += gridDim.x) {
            const bool first = tile == (int)blockIdx.x;
            const int k0 = kstart + tile * KT, k1 = min(L, k0 + KT), n = k1 - k0;
            uint16_t* Kt = reinterpret_cast<uint16_t*>(abuf);
            uint16_t* Vt = Kt + (size_t)KT * hd;
            if (threadIdx.x == 0) {
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&wbar[2], (uint32_t)(2 * n * hd * 2));
                bulk_load(Kt, ly.kc + (size_t)k0 * hd, n * hd * 2, &wbar[2]);
                bulk_load(Vt, ly.vc + (size_t)k0 * hd, n * hd * 2, &wbar[2]);
            }
            pend[2] = true;
            if (first) mark();  // K/V tile requested
            const bool last = k1 == L;
            float* kv_new = p_s + 8 * KT;  // [2][hd] after the probabilities
            // q once per layer; k and v (slots heads, heads + 1) for the tile holding the position
            const int s0 = have_q ? P.heads : 0, s1 = P.heads + ((last && ly.has_kv) ? 2 : 0);
            if (s0 < s1) {
                const float* rope = rope_s + (ly.full ? 512 : 0);
                if (hd == 256)
                    qkv_slots<256>(pq, ly, P.heads, P.eps, s0, s1, rope, q_s, kv_new);
                else
                    qkv_slots<512>(pq, ly, P.heads, P.eps, s0, s1, rope, q_s, kv_new);
            }
            have_q = true;
            if (first) mark();  // q (and k, v) ready
            if (!(ok = copy_wait(2, 0x53))) break;
            if (first) mark();  // K/V tile in shared memory
            if (last && ly.has_kv) {  // append the new position (KVCache.append) and use it
                for (int i = threadIdx.x; i < hd; i += kThreads) {
                    const uint16_t kb = (uint16_t)f32_to_bf16_bits(kv_new[i]);
                    const uint16_t vb = (uint16_t)f32_to_bf16_bits(kv_new[hd + i]);
                    Kt[(size_t)(pos - k0) * hd + i] = kb;
                    Vt[(size_t)(pos - k0) * hd + i] = vb;
                    ly.kc[(size_t)pos * hd + i] = kb;
                    ly.vc[(size_t)pos * hd + i] = vb;
                }
            }
            __syncthreads();
            float* part = P.attn_part + (size_t)tile * P.heads * (hd + 2);
            if (hd == 256)
                attend_tile<256>(Kt, Vt, n, P.heads, q_s, p_s, part);
            else
                attend_tile<512>(Kt, Vt, n, P.heads, q_s, p_s, part);
            __syncthreads();
            if (first) mark();  // tile done
        }
        if (!ok) break;
        if ((int)blockIdx.x >= ntile)
            for (int k = 0; k < 4; ++k) mark();  // no tile: the four attention stamps at once
        if (!(ok = grid_sync(gr, s_flag, 0x54))) break;
        // ---- combine (each CTA a slice of the outputs), o projection, post-attention norm +
        // residual, pre-MLP norm ----
        {
            // staging in the q/k/v buffer (idle until the gate/up prefetch, requested later)
            float* ml = reinterpret_cast<float*>(abuf);
            if (hd == 256)
                combine_tiles<256>(P.attn_part, ntile, P.heads, ml, red, p_s, P.attn_out);
            else
                combine_tiles<512>(P.attn_part, ntile, P.heads, ml, red, p_s, P.attn_out);
            mark();
        }
        if (!(ok = grid_sync(gr, s_flag, 0x55))) break;
        load_x(x_s, P.attn_out, P.heads * hd);
        mark();
        if (!(ok = compute_weights(wcur++))) break;
        if (!(ok = grid_sync(gr, s_flag, 0x56))) break;
        post_norm_add(sph[ly.wo], h_s, ly.n_pa, 1.f, ly.n_pf, H, P.eps, x_s, sred,
                      reinterpret_cast<float*>(wbuf[ly.wo & 1]));
        mark();
        // ---- gate/up with GeGLU ----
        if (!(ok = compute_weights(wcur++))) break;
        if (!(ok = grid_sync(gr, s_flag, 0x57))) break;
        // ---- down, post-FFN norm + residual ----
        load_x(x_s, sph[ly.wgu].act, ly.inter);
        mark();
        if (!(ok = compute_weights(wcur++))) break;
        if (!(ok = grid_sync(gr, s_flag, 0x58))) break;
        post_norm_add(sph[ly.wd], h_s, ly.n_pff, 1.f, nullptr, H, P.eps, x_s, sred,
                      reinterpret_cast<float*>(wbuf[ly.wd & 1]));
        mark();
        // ---- PLE gate ----
        if (!(ok = compute_weights(wcur++))) break;
        if (!(ok = grid_sync(gr, s_flag, 0x59))) break;
        // ---- per-layer input (PLE mix) and GELU gate: pa = bf16(gelu(pg) * per_layer[l]) ----
        {
            const int PD = P.pdim;  // PD <= kThreads: thread owns element d (this CTA's rotated order)
            int d = threadIdx.x;
            if (d < PD) {
                d += rot_of(PD);
                if (d >= PD) d -= PD;
            }
            const WPhase& ppg = sph[ly.wpg];
            float* pvs = reinterpret_cast<float*>(wbuf[ly.wpg & 1]);  // idle until the next prefetch
            float pv = 0.f, pg = 0.f, pn = 0.f, tok = 0.f;
            if ((int)threadIdx.x < PD) {  // every load of the element first
                const int col = l * PD + d;
                pv = plane_sum(top, col) * P.proj_scale;  // proj * (1 / sqrt(hidden)), gemma4-webgpu.js:319-320
                pg = plane_sum(ppg, d);
                pn = __ldg(P.ple_norm + d);
                if (id_ok) {
                    const uint8_t byte = __ldg(P.ple_packed + (size_t)id * (P.ple_width / 2) + (col >> 1));
                    const int nib = (col & 1) ? (byte >> 4) : (byte & 0xF);
                    const float sc =
                        bf16_bits_to_f32(__ldg(P.ple_scales + (size_t)id * (P.ple_width / 32) + (col >> 5)));
                    tok = (float)(nib >= 8 ? nib - 16 : nib) * sc;
                }
            }
            if ((int)threadIdx.x < PD) pvs[d] = pv;
            __syncthreads();
            const float pvf = (int)threadIdx.x < PD ? pvs[threadIdx.x] : 0.f;  // fixed order for the sum
            const float inv = rsqrtf(block_sum(pvf * pvf, sred) / (float)PD + P.eps);
            if ((int)threadIdx.x < PD) {
                const float per = (pv * inv * pn + tok * sqrtf((float)PD)) * 0.7071067811865476f;
                x_s[d] = (uint16_t)f32_to_bf16_bits(gelu_ref(pg) * per);
            }
            __syncthreads();
            mark();
        }
        // ---- PLE projection, post-PLE norm + residual * skip, next layer's input norm ----
        if (!(ok = compute_weights(wcur++))) break;
        if (!(ok = grid_sync(gr, s_flag, 0x5A))) break;
        post_norm_add(sph[ly.wpp], h_s, ly.n_pple, ly.skip, ly.w_next, H, P.eps, x_s, sred,
                      reinterpret_cast<float*>(wbuf[ly.wpp & 1]));
        mark();
    }

    // ---- tied bf16 LM head, softcap, greedy pick (BF16_HEAD :1265-1277, gemma4-webgpu.js:441-480) ----
    if (ok) {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        const int r0 = (int)((long long)P.vocab * blockIdx.x / gridDim.x);
        const int r1 = (int)((long long)P.vocab * (blockIdx.x + 1) / gridDim.x);
        // this CTA's vocabulary rows stream through four half-buffer stages (the weight buffers
        // are idle once the last linear is done), head_rows rows each, one mbarrier per stage
        const int R = P.head_rows;
        const int nst = (r1 - r0 + R - 1) / R;
        const size_t half = (size_t)R * H * 2;
        uint8_t* stage[4] = {wbuf[0], wbuf[0] + half, wbuf[1], wbuf[1] + half};
        const int sbar[4] = {0, 3, 1, 4};
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        uint4 xr[kMaxH / 256];  // this lane's columns lane*8 + 256c of x
#pragma unroll
        for (int c = 0; c < kMaxH / 256; ++c)
            xr[c] = lane * 8 + 256 * c < H ? *reinterpret_cast<const uint4*>(x_s + lane * 8 + 256 * c)
                                           : make_uint4(0, 0, 0, 0);
        auto issue_stage = [&](int s) -> bool {
            if (s >= nst) return false;
            const int a = r0 + s * R, rows = min(R, r1 - a);
            const int b = sbar[s & 3];
            if (threadIdx.x == 0) {
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&wbar[b], (uint32_t)(rows * H * 2));
                bulk_load(stage[s & 3], P.embed + (size_t)a * H, rows * H * 2, &wbar[b]);
            }
            return true;
        };
        for (int b = 0; b < 2 && ok; ++b)
            if (pend[b]) ok = copy_wait(b, 0x5B);
        for (int s = 0; s < 4 && ok; ++s) pend[sbar[s]] = issue_stage(s);
        for (int s = 0; s < nst && ok; ++s) {
            const int b = sbar[s & 3];
            if (!(ok = copy_wait(b, 0x5C))) break;
            const int a = r0 + s * R, rows = min(R, r1 - a);
            const uint16_t* W = reinterpret_cast<const uint16_t*>(stage[s & 3]);
            for (int r = warp; r < rows; r += kWarps) {
                float acc = 0.f;
#pragma unroll
                for (int c = 0; c < kMaxH / 256; ++c) {
                    if (lane * 8 + 256 * c >= H) break;
                    const uint4 wv = *reinterpret_cast<const uint4*>(W + (size_t)r * H + lane * 8 + 256 * c);
                    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
                    const uint32_t xx[4] = {xr[c].x, xr[c].y, xr[c].z, xr[c].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        acc = fmaf(lo_bf16(ww[e]), lo_bf16(xx[e]), acc);
                        acc = fmaf(hi_bf16(ww[e]), hi_bf16(xx[e]), acc);
                    }
                }
                acc = warp_sum(acc);
                const float capped = P.softcap > 0.f ? tanhf(acc / P.softcap) * P.softcap : acc;
                const int idx = a + r;
                if (capped > bv || (capped == bv && idx < bi)) {  // lowest index among equal maxima
                    bv = capped;
                    bi = idx;
                }
            }
            __syncthreads();  // the stage is refilled next
            pend[b] = issue_stage(s + 4);
        }
        // CTA best: warps -> red
        if (ok) {
            if (lane == 0) {
                red[warp * 2] = bv;
                reinterpret_cast<int*>(red)[warp * 2 + 1] = bi;
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                float v = red[0];
                int ix = reinterpret_cast<int*>(red)[1];
                for (int w = 1; w < kWarps; ++w) {
                    const float v2 = red[w * 2];
                    const int i2 = reinterpret_cast<int*>(red)[w * 2 + 1];
                    if (v2 > v || (v2 == v && i2 < ix)) {
                        v = v2;
                        ix = i2;
                    }
                }
                P.head_part[blockIdx.x] = make_float2(v, __int_as_float(ix));
            }
            ok = grid_sync(gr, s_flag, 0x5D);
        }
        if (ok && blockIdx.x == 0 && threadIdx.x == 0) {
            float v = -INFINITY;
            int ix = 0x7fffffff;
            for (unsigned c = 0; c < gridDim.x; ++c) {
                const float2 pc = __ldcg(P.head_part + c);
                const int i2 = __float_as_int(pc.y);
                if (pc.x > v || (pc.x == v && i2 < ix)) {
                    v = pc.x;
                    ix = i2;
                }
            }
            P.next[0] = ix;
            if (P.val) P.val[0] = v;
            P.seq_pos[0] = pos + 1;
        }
    }

    // ---- leave: wait for this CTA's copies still in flight ----
    for (int b = 0; b < kBars; ++b)
        if (pend[b]) {
            mbar_wait(&wbar[b], par[b], P.err, 0x5E);
            par[b] ^= 1u;
        }
    mark();
}

}  // namespace

// ----------------------------------------------------------------------- host ----

struct g4_decoder {
    g4_ctx* ctx = nullptr;
    DParams p{};
    std::vector<WPhase> ph;
    std::vector<DLayer> layers;
    WPhase* d_ph = nullptr;
    DLayer* d_layers = nullptr;
    std::vector<void*> allocs;
    int smem = 0;
    int grid = 0;
};

namespace {

g4_status dec_alloc(g4_decoder* d, void** p, size_t bytes) {
    G4_CHECK_CUDA(cudaMalloc(p, bytes));
    d->allocs.push_back(*p);
    G4_CHECK_CUDA(cudaMemsetAsync(*p, 0, bytes, d->ctx->stream));
    return G4_OK;
}

// A weight phase for linear `lin`: split K until there are about two units per CTA (S <= 8,
// >= 4 blocks per unit), partial planes [S][N]; GeGLU phases keep whole K (the epilogue needs
// the sums).
g4_status make_phase(g4_decoder* d, const g4_linear* lin, int K, int N, int kind, int grid, WPhase* out,
                     int* max_bytes) {
    if (!lin) return g4::set_error(G4_ERR_INVALID, "g4_decoder_create: null linear");
    const g4_linear_dev& L = lin->dev;
    if (L.K != K || L.N != N)
        return g4::set_error(G4_ERR_INVALID, "g4_decoder_create: linear is %d x %d, the model wants %d x %d", L.K, L.N,
                             K, N);
    if (K % 64 != 0 || N % 16 != 0)
        return g4::set_error(G4_ERR_UNSUPPORTED, "g4_decoder_create: K %d / N %d (multiples of 64 / 16)", K, N);
    WPhase w{};
    w.wfrag = L.wfrag;
    w.sfrag = L.sfrag;
    w.K = K;
    w.N = N;
    w.Kc = L.Kc;
    w.NT = L.NT;
    w.kind = kind;
    int per_unit_blocks;
    if (kind == kGeglu) {
        if (N % 128 != 0) return g4::set_error(G4_ERR_UNSUPPORTED, "g4_decoder_create: gate/up N %d", N);
        w.S = 1;
        w.bpu = w.Kc;
        w.units = N / 32;  // (slab, i): 4 pairs of 16-row tiles per 128-row slab
        per_unit_blocks = 2 * w.Kc;
        g4_status st = dec_alloc(d, reinterpret_cast<void**>(&w.act), (size_t)(N / 2) * 2);
        if (st) return st;
    } else {
        int S = 1;
        while (S < kMaxSplits && w.NT * S < 2 * grid && (w.Kc + 2 * S - 1) / (2 * S) >= 4) S *= 2;
        w.bpu = (w.Kc + S - 1) / S;
        w.S = (w.Kc + w.bpu - 1) / w.bpu;
        w.units = w.NT * w.S;
        per_unit_blocks = w.bpu;
        g4_status st = dec_alloc(d, reinterpret_cast<void**>(&w.planes), (size_t)w.S * N * 4);
        if (st) return st;
    }
    const int units_per_cta = (w.units + grid - 1) / grid;
    *max_bytes = std::max(*max_bytes, units_per_cta * per_unit_blocks * (kBlockW + kBlockS));
    *out = w;
    return G4_OK;
}

}  // namespace

extern "C" {

g4_status g4_decoder_create(g4_ctx* ctx, const g4_decoder_desc* desc, const g4_decoder_layer* layers,
                            g4_decoder** out) {
    if (!out) return g4::set_error(G4_ERR_INVALID, "g4_decoder_create: null out");
    *out = nullptr;
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!desc || !layers || !desc->top || !desc->embed || !desc->ple || !desc->ple_norm || !desc->final_norm)
        return g4::set_error(G4_ERR_INVALID, "g4_decoder_create: null argument");
    const int Lc = desc->layers, H = desc->hidden, heads = desc->heads, PD = desc->ple_dim;
    if (Lc < 1 || H < 256 || H > kMaxH || H % 256 != 0 || heads < 1 || heads > 8 || PD < 32 || PD > kThreads ||
        PD % 32 != 0 || desc->window < 1)
        return g4::set_error(G4_ERR_UNSUPPORTED,
                             "g4_decoder_create: layers %d hidden %d heads %d ple_dim %d window %d outside the "
                             "persistent decoder's range",
                             Lc, H, heads, PD, desc->window);
    if (desc->ple->width != Lc * PD)
        return g4::set_error(G4_ERR_INVALID, "g4_decoder_create: PLE width %d != layers x ple_dim", desc->ple->width);
    if (desc->embed->K != H || desc->embed->N != desc->vocab || desc->vocab < 1 || desc->ple->vocab < desc->vocab)
        return g4::set_error(G4_ERR_INVALID,
                             "g4_decoder_create: embedding [%d, %d] and PLE table of %d rows for vocab %d, hidden %d",
                             desc->embed->N, desc->embed->K, desc->ple->vocab, desc->vocab, H);
    const void* emb = desc->embed->w;

    g4_decoder* d = new g4_decoder();
    d->ctx = ctx;
    const int grid = ctx->num_sms;
    d->grid = grid;
    int max_bytes = 0, kmax = H, hdmax = 0, cap = 1 << 30;
    bool rope_set[2] = {false, false};
    int rope_hd[2] = {256, 256}, rope_n[2] = {0, 0};
    float rope_base[2] = {10000.f, 10000.f};
    d->ph.resize(1 + 6 * Lc);
    d->layers.resize(Lc);
    auto fail = [&](g4_status s) {
        g4_decoder_destroy(d);
        return s;
    };
    st = make_phase(d, desc->top, H, Lc * PD, kPlanes, grid, &d->ph[0], &max_bytes);
    if (st) return fail(st);
    for (int l = 0; l < Lc; ++l) {
        const g4_decoder_layer& a = layers[l];
        DLayer& y = d->layers[l];
        if (!a.kv || !a.n_in || !a.n_pa || !a.n_pf || !a.n_pff || !a.n_pple || !a.qn || (a.has_kv && !a.kn))
            return fail(g4::set_error(G4_ERR_INVALID, "g4_decoder_create: layer %d: null argument", l));
        int len = 0, hd = 0, kcap = 0;
        void *kb = nullptr, *vb = nullptr;
        g4_kv_info(a.kv, &len, &hd, &kcap);
        g4_kv_buffers(a.kv, &kb, &vb);
        int ring = 0;
        g4_kv_layout(a.kv, &ring, nullptr, nullptr);
        if (ring)  // the decoder addresses keys by position
            return fail(g4::set_error(G4_ERR_UNSUPPORTED, "g4_decoder_create: layer %d has a ring KV cache", l));
        if (hd != 256 && hd != 512)
            return fail(g4::set_error(G4_ERR_UNSUPPORTED, "g4_decoder_create: layer %d head dim %d", l, hd));
        if (a.inter < 64 || a.inter % 64 != 0)
            return fail(g4::set_error(G4_ERR_UNSUPPORTED, "g4_decoder_create: layer %d MLP width %d", l, a.inter));
        const int w0 = 1 + 6 * l;
        const int qn = heads * hd + (a.has_kv ? 2 * hd : 0);
        if ((st = make_phase(d, a.qkv, H, qn, kPlanes, grid, &d->ph[w0 + 0], &max_bytes))) return fail(st);
        if ((st = make_phase(d, a.o, heads * hd, H, kPlanes, grid, &d->ph[w0 + 1], &max_bytes))) return fail(st);
        if ((st = make_phase(d, a.gu, H, 2 * a.inter, kGeglu, grid, &d->ph[w0 + 2], &max_bytes))) return fail(st);
        if ((st = make_phase(d, a.down, a.inter, H, kPlanes, grid, &d->ph[w0 + 3], &max_bytes))) return fail(st);
        if ((st = make_phase(d, a.pg, H, PD, kPlanes, grid, &d->ph[w0 + 4], &max_bytes))) return fail(st);
        if ((st = make_phase(d, a.pp, PD, H, kPlanes, grid, &d->ph[w0 + 5], &max_bytes))) return fail(st);
        y.wq = w0;
        y.wo = w0 + 1;
        y.wgu = w0 + 2;
        y.wd = w0 + 3;
        y.wpg = w0 + 4;
        y.wpp = w0 + 5;
        y.n_pa = a.n_pa;
        y.n_pf = a.n_pf;
        y.n_pff = a.n_pff;
        y.n_pple = a.n_pple;
        y.qn = a.qn;
        y.kn = a.kn;
        y.w_next = l + 1 < Lc ? layers[l + 1].n_in : desc->final_norm;
        y.skip = a.skip;
        y.kc = static_cast<uint16_t*>(kb);
        y.vc = static_cast<uint16_t*>(vb);
        y.hd = hd;
        y.full = a.full ? 1 : 0;
        y.has_kv = a.has_kv ? 1 : 0;
        y.rope_angles = a.rope_angles;
        y.rope_base = a.rope_base;
        y.inter = a.inter;
        // one RoPE table per layer kind: every layer of a kind must share (hd, base, pairs)
        if (a.rope_angles < 0 || a.rope_angles > hd / 2)
            return fail(g4::set_error(G4_ERR_INVALID, "g4_decoder_create: layer %d rope_angles %d", l, a.rope_angles));
        const int kind = y.full;
        if (!rope_set[kind]) {
            rope_set[kind] = true;
            rope_hd[kind] = hd;
            rope_n[kind] = a.rope_angles;
            rope_base[kind] = a.rope_base;
        } else if (rope_hd[kind] != hd || rope_n[kind] != a.rope_angles || rope_base[kind] != a.rope_base) {
            return fail(g4::set_error(G4_ERR_UNSUPPORTED, "g4_decoder_create: layer %d RoPE differs from its kind", l));
        }
        kmax = std::max(kmax, std::max(heads * hd, a.inter));
        hdmax = std::max(hdmax, hd);
        cap = std::min(cap, kcap);
        if (kcap > kMaxTiles * (16384 / hd))
            return fail(g4::set_error(G4_ERR_UNSUPPORTED, "g4_decoder_create: layer %d cache of %d rows (max %d)", l,
                                      kcap, kMaxTiles * (16384 / hd)));
    }
    // the combine gives each CTA heads x hd / grid <= kThreads outputs
    if ((heads * hdmax + grid - 1) / grid > kThreads)
        return fail(g4::set_error(G4_ERR_UNSUPPORTED, "g4_decoder_create: %d attention outputs over %d CTAs",
                                  heads * hdmax, grid));
    // shared memory plan
    DParams& p = d->p;
    const int att_tile = 2 * 16384 * 2;  // K and V tiles of 16384 / hd keys (also >= the combine's staging)
    static_assert(2 * 16384 * 2 >= 2 * kMaxTiles * 8 * 4, "combine staging fits the attention buffer");
    int wb = std::max(max_bytes, att_tile);
    wb = (wb + 127) & ~127;
    int off = 0;
    auto take = [&](int bytes) {
        const int o = off;
        off += (bytes + 127) & ~127;
        return o;
    };
    p.off_bar = take(kBars * 8);
    p.off_h = take(H * 4);
    p.off_x = take(kmax * 2);
    p.off_q = take(heads * hdmax * 4);
    p.off_p = take((8 * 64 + 2 * hdmax) * 4);  // probabilities [16384/hd keys][8] + new k, v; combine denominators
    p.off_red = take(kWarps * 2 * 2 * 32 * 4);
    p.off_sred = take(64 * 4);
    p.off_ph = take((int)(d->ph.size() * sizeof(WPhase)));
    p.off_ly = take((int)(d->layers.size() * sizeof(DLayer)));
    p.off_rope = take(2 * 512 * 4);
    p.off_w0 = take(0);
    p.wbuf = wb;
    const int smem = p.off_w0 + 2 * wb;
    if (smem > kMaxSmem)
        return fail(g4::set_error(G4_ERR_UNSUPPORTED,
                                  "g4_decoder_create: %d bytes of shared memory per CTA needed (max %d): a linear "
                                  "share of %d bytes is too large",
                                  smem, kMaxSmem, max_bytes));
    p.head_rows = wb / 2 / (H * 2);  // half a buffer per stage: >= 16 rows (wb >= 64 KB, H <= 2048)
    p.L = Lc;
    p.nph = (int)d->ph.size();
    for (int k = 0; k < 2; ++k) {
        p.rope_hd[k] = rope_hd[k];
        p.rope_n[k] = rope_n[k];
        p.rope_base[k] = rope_base[k];
    }
    p.H = H;
    p.heads = heads;
    p.pdim = PD;
    p.vocab = desc->vocab;
    p.window = desc->window;
    p.cap = cap;
    p.eps = desc->eps;
    p.softcap = desc->softcap;
    p.proj_scale = (float)(1.0 / sqrt((double)H));
    p.embed = static_cast<const uint16_t*>(emb);
    p.ple_packed = desc->ple->packed;
    p.ple_scales = desc->ple->scales;
    p.ple_width = desc->ple->width;
    p.ple_norm = desc->ple_norm;
    p.n_in0 = layers[0].n_in;
    if ((st = dec_alloc(d, reinterpret_cast<void**>(&p.attn_part), (size_t)kMaxTiles * heads * (hdmax + 2) * 4)))
        return fail(st);
    if ((st = dec_alloc(d, reinterpret_cast<void**>(&p.attn_out), (size_t)heads * hdmax * 2))) return fail(st);
    if ((st = dec_alloc(d, reinterpret_cast<void**>(&p.head_part), (size_t)grid * sizeof(float2)))) return fail(st);
    if ((st = dec_alloc(d, reinterpret_cast<void**>(&p.sync), kSyncBytes))) return fail(st);
    if ((st = dec_alloc(d, reinterpret_cast<void**>(&d->d_ph), d->ph.size() * sizeof(WPhase)))) return fail(st);
    if ((st = dec_alloc(d, reinterpret_cast<void**>(&d->d_layers), d->layers.size() * sizeof(DLayer))))
        return fail(st);
    cudaError_t e = cudaMemcpyAsync(d->d_ph, d->ph.data(), d->ph.size() * sizeof(WPhase), cudaMemcpyHostToDevice,
                                    ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d->d_layers, d->layers.data(), d->layers.size() * sizeof(DLayer), cudaMemcpyHostToDevice,
                            ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return fail(g4::cuda_error(e, "g4_decoder_create: upload"));
    p.ph = d->d_ph;
    p.layers = d->d_layers;
    p.err = ctx->d_err;
    d->smem = smem;
    e = cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return fail(g4::cuda_error(e, "g4_decoder_create: shared memory attribute"));
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel, kThreads, smem);
    if (e != cudaSuccess || per_sm < 1)
        return fail(g4::set_error(G4_ERR_UNSUPPORTED, "g4_decoder_create: the step kernel does not fit an SM"));
    *out = d;
    return G4_OK;
}

g4_status g4_decoder_destroy(g4_decoder* dec) {
    if (!dec) return G4_OK;
    if (dec->ctx) {
        cudaSetDevice(dec->ctx->device);
        cudaStreamSynchronize(dec->ctx->stream);
    }
    for (void* p : dec->allocs) cudaFree(p);
    delete dec;
    return G4_OK;
}

g4_status g4_decoder_reset(g4_decoder* dec) {
    if (!dec) return g4::set_error(G4_ERR_INVALID, "g4_decoder_reset: null decoder");
    g4_status st = g4::use_device(dec->ctx);
    if (st) return st;
    G4_CHECK_CUDA(cudaStreamSynchronize(dec->ctx->stream));
    G4_CHECK_CUDA(cudaMemset(dec->p.sync, 0, kSyncBytes));
    return G4_OK;
}

g4_status g4_decoder_set_timeline(g4_decoder* dec, unsigned long long* timeline, int entries) {
    if (!dec) return g4::set_error(G4_ERR_INVALID, "g4_decoder_set_timeline: null decoder");
    if (timeline && entries < 2) return g4::set_error(G4_ERR_INVALID, "g4_decoder_set_timeline: %d entries", entries);
    dec->p.timeline = timeline;
    dec->p.timeline_cap = timeline ? entries : 0;
    return G4_OK;
}

g4_status g4_decoder_step(g4_ctx* ctx, g4_decoder* dec, const int32_t* ids, int32_t* seq_pos, int32_t* next,
                          float* val) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!dec || !ids || !seq_pos || !next) return g4::set_error(G4_ERR_INVALID, "g4_decoder_step: null argument");
    if (dec->ctx->device != ctx->device)
        return g4::set_error(G4_ERR_INVALID, "g4_decoder_step: decoder of device %d on device %d", dec->ctx->device,
                             ctx->device);
    DParams p = dec->p;
    p.ids = ids;
    p.seq_pos = seq_pos;
    p.next = next;
    p.val = val;
    p.err = ctx->d_err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(dec->grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = dec->smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_step_kernel, p);
    if (e != cudaSuccess) return g4::cuda_error(e, "g4_decoder_step: launch");
    g4::count_launch();
    return G4_OK;
}

}  // extern "C"
