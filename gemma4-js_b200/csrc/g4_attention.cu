// g4_attention.cu -- bf16 KV cache and GQA decode attention (flash-decoding on B200).
//
// The reference runs attention as three WGSL dispatches with the logits and
// probabilities materialised in global memory and a softmax of one thread per row
// (custom-webgpu/gpu-runtime.js:1204-1248, :1357-1365).  Here one kernel streams the
// bf16 K/V tiles through shared memory with TMA (128B-swizzled boxes, mbarrier
// pipeline, one producer warp), computes S^T = K Q^T and O^T += V^T P^T on the tensor
// cores with the 8 query heads as the n = 8 dimension (so no padding is computed),
// and keeps an online softmax in registers.  Long key ranges are split over CTAs
// (split-KV) and merged by a small combine kernel through a scratch buffer.  Batched
// decode of a sliding layer with more sequences than SMs uses tiles of half the keys so
// that two CTAs share an SM: every CTA of the grid is resident from the start and no
// second wave starts cold behind the first.
#include <stdio.h>

#include <algorithm>
#include <mutex>

#include "g4_attention.cuh"
#include "g4_common.cuh"

namespace {

using namespace g4dev;

constexpr float kLog2e = 1.4426950408889634f;

template <int HD, bool kNarrow = false>
struct AttnCfg {
    static constexpr int KT = (kNarrow ? 8192 : 16384) / HD;  // keys per pipeline stage
    static constexpr int WARPS = KT / 16;       // consumer warps, 16 keys each
    static constexpr int BOXES = HD / 64;       // 128-byte wide TMA boxes per row
    static constexpr int BOX_BYTES = KT * 128;  // one box: KT rows x 128 B
    static constexpr int TILE_BYTES = KT * HD * 2;
    static constexpr int STAGES = 3;
    static constexpr int SMEM = STAGES * 2 * TILE_BYTES + 1024 + 256;
    static constexpr int THREADS = (WARPS + 1) * 32;
    static constexpr int CTAS_PER_SM = kNarrow ? 2 : 1;
};

// Smem address of (key, d) for ldmatrix in a 128B-swizzled [KT x HD] tile.
template <class C>
__device__ __forceinline__ uint32_t tile_addr(uint32_t base, int key, int d) {
    const int box = d >> 6, chunk = (d & 63) >> 3;
    return base + box * C::BOX_BYTES + key * 128 + (((chunk ^ (key & 7))) << 4);
}

struct AttnParams {
    const uint16_t* q;      // [rows, heads, hd]
    uint16_t* out;          // [rows, heads, hd]
    float* part_o;          // [rows, nsplit, 8, hd]   (nsplit > 1)
    float2* part_ml;        // [rows, nsplit, 8]       (nsplit > 1)
    uint32_t* err;
    int heads, keylen, qpos0, sliding, window;
    int ring;                // ring cache: key j sits in row kv_row0 + j % ring (mirrored past the ring)
    int nsplit, split_keys;  // keys per split (multiple of KT)
    int kv_row0;             // first cache row of this sequence in the tensor map
    // Device-side positions (g4_rows): when seq_pos is set, row r belongs to sequence
    // seq = seq_base + r / rows_per_seq, sits at seq_pos[seq] + pos0 + r % rows_per_seq,
    // sees keylen = seq_pos[seq] + pos0 + rows_per_seq keys, and the sequence's cache
    // rows start at seq * seq_stride.
    const int32_t* seq_pos;
    int seq_base, rows_per_seq, pos0, seq_stride;
    // G4_ROWS_HISTORY_READY: seq_pos and the cache rows below each row's first position
    // are final before this grid starts, so they are read before the PDL wait.
    int history_ready;
};

template <int HD, bool kNarrow>
__global__ void __launch_bounds__(AttnCfg<HD, kNarrow>::THREADS, AttnCfg<HD, kNarrow>::CTAS_PER_SM)
attn_decode_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   AttnParams p) {
    using C = AttnCfg<HD, kNarrow>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // Offset the __shared__ array itself (not an integer round trip) so the compiler keeps
    // shared-memory addressing for every access through `smem`.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* kst = smem;                                   // [STAGES][TILE]
    uint8_t* vst = smem + C::STAGES * C::TILE_BYTES;       // [STAGES][TILE]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * C::STAGES * C::TILE_BYTES);
    uint64_t* empty = full + C::STAGES;

    pdl_trigger();
    // q and the K/V rows of the current positions come from the predecessors.  With
    // history_ready the older rows (and the positions) are final already: the producer
    // streams them while the predecessors drain and waits only before the first tile
    // that reaches the current positions.
    const bool early = p.history_ready && p.seq_pos;
    if (!early) pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.y, split = blockIdx.x;
    int qp, keylen, kv_row0, first_new = 0;
    if (p.seq_pos) {
        const int seq = p.seq_base + r / p.rows_per_seq;
        const int base = p.seq_pos[seq] + p.pos0;
        first_new = base;
        qp = base + r % p.rows_per_seq;
        keylen = base + p.rows_per_seq;
        kv_row0 = seq * p.seq_stride;
    } else {
        qp = p.qpos0 + r;
        keylen = p.keylen;
        kv_row0 = p.kv_row0;
    }
    const int hi = min(qp, keylen - 1);
    const int lo = p.sliding ? max(0, qp - p.window + 1) : 0;
    const int s_lo = lo + split * p.split_keys;
    const int s_hi = min(hi, s_lo + p.split_keys - 1);  // inclusive
    const int nkeys = s_hi >= s_lo ? s_hi - s_lo + 1 : 0;
    const int ntiles = (nkeys + C::KT - 1) / C::KT;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], C::WARPS);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == C::WARPS) {
        // ------------------------------------------------ TMA producer warp --
        if (lane == 0 && ntiles > 0) {
            prefetch_tensor_map(&kmap);
            prefetch_tensor_map(&vmap);
            bool ok = true, waited = !early;
            for (int t = 0; t < ntiles && ok; ++t) {
                if (!waited && s_lo + (t + 1) * C::KT > first_new) {  // the tile reaches the current rows
                    pdl_wait();
                    waited = true;
                }
                const int s = t % C::STAGES;
                if (t >= C::STAGES) ok = mbar_wait(&empty[s], ((t / C::STAGES) - 1) & 1, p.err);
                if (!ok) break;
                mbar_arrive_expect_tx(&full[s], 2 * C::TILE_BYTES);
                const int j0 = s_lo + t * C::KT;
                const int y = kv_row0 + (p.ring ? j0 % p.ring : j0);
#pragma unroll
                for (int b = 0; b < C::BOXES; ++b) {
                    tma_load_2d(kst + s * C::TILE_BYTES + b * C::BOX_BYTES, &kmap, &full[s], b * 64, y);
                    tma_load_2d(vst + s * C::TILE_BYTES + b * C::BOX_BYTES, &vmap, &full[s], b * 64, y);
                }
            }
            // Drain: do not leave while our copies may still be landing.
            const int first = ntiles > C::STAGES ? ntiles - C::STAGES : 0;
            for (int t = first; t < ntiles; ++t) mbar_wait(&full[t % C::STAGES], (t / C::STAGES) & 1, p.err);
        }
        // The producer warp still takes part in the final __syncthreads below.
    }

    const int g = lane >> 2, tq = lane & 3;
    float o[HD / 16][4];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
#pragma unroll
    for (int i = 0; i < HD / 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

    if (early) pdl_wait();  // every thread waits (the producer's lane 0 again: a no-op)
    if (warp < C::WARPS) {
        // Q^T as the B operand: b0b1 = Q[head g][16ks + 2tq ..], b2b3 = Q[g][16ks + 8 + 2tq ..]
        uint32_t qf[HD / 16][2];
        const uint32_t* qrow = reinterpret_cast<const uint32_t*>(p.q + ((size_t)r * p.heads + g) * HD);
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
            qf[ks][0] = g < p.heads ? __ldg(qrow + ks * 8 + tq) : 0u;
            qf[ks][1] = g < p.heads ? __ldg(qrow + ks * 8 + 4 + tq) : 0u;
        }
        const int j = lane >> 3, rr = lane & 7;
        for (int t = 0; t < ntiles; ++t) {
            const int s = t % C::STAGES;
            if (!mbar_wait(&full[s], (t / C::STAGES) & 1, p.err)) break;
            const uint32_t kb = smem_u32(kst + s * C::TILE_BYTES);
            const uint32_t vb = smem_u32(vst + s * C::TILE_BYTES);
            // ---- S^T[16 keys x 8 heads] = K Q^T ----
            float sc[4] = {0.f, 0.f, 0.f, 0.f};
            {
                const int key = warp * 16 + ((j & 1) << 3) + rr;
#pragma unroll
                for (int ks = 0; ks < HD / 16; ++ks) {
                    uint32_t a[4];
                    ldmatrix_x4(a, tile_addr<C>(kb, key, ks * 16 + ((j >> 1) << 3)));
                    const uint32_t b[2] = {qf[ks][0], qf[ks][1]};
                    mma_bf16_16816(sc, a, b, sc);
                }
            }
            // ---- mask (QK_SHADER :1214-1217) and online softmax, base 2 ----
            const int key0 = s_lo + t * C::KT + warp * 16 + g;
            const bool v0 = key0 <= s_hi, v1 = key0 + 8 <= s_hi;
            float x0 = v0 ? sc[0] * kLog2e : -INFINITY, x1 = v0 ? sc[1] * kLog2e : -INFINITY;
            float x2 = v1 ? sc[2] * kLog2e : -INFINITY, x3 = v1 ? sc[3] * kLog2e : -INFINITY;
            float mt0 = fmaxf(x0, x2), mt1 = fmaxf(x1, x3);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, off));
                mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, off));
            }
            const float mn0 = fmaxf(m0, mt0), mn1 = fmaxf(m1, mt1);
            const float mu0 = mn0 == -INFINITY ? 0.f : mn0, mu1 = mn1 == -INFINITY ? 0.f : mn1;
            const float al0 = exp2f(m0 - mu0), al1 = exp2f(m1 - mu1);
            const float p0 = exp2f(x0 - mu0), p1 = exp2f(x1 - mu1);
            const float p2 = exp2f(x2 - mu0), p3 = exp2f(x3 - mu1);
            l0 = l0 * al0 + p0 + p2;
            l1 = l1 * al1 + p1 + p3;
            m0 = mn0;
            m1 = mn1;
            if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
                for (int i = 0; i < HD / 16; ++i) {
                    o[i][0] *= al0;
                    o[i][1] *= al1;
                    o[i][2] *= al0;
                    o[i][3] *= al1;
                }
            }
            // ---- P^T as the B operand: transpose the two 8x8 key blocks.  P is split
            // into a bf16 head and a bf16 tail (P = hi + lo to ~2^-16), so the P.V
            // products keep almost f32 precision; the tensor cores have room for the
            // second mma in this HBM-bound loop. ----
            const uint32_t h01 = pack_bf16x2_bits(p0, p1), h23 = pack_bf16x2_bits(p2, p3);
            const uint32_t l01 = pack_bf16x2_bits(p0 - bf16_bits_to_f32(h01 & 0xFFFFu), p1 - bf16_bits_to_f32(h01 >> 16));
            const uint32_t l23 = pack_bf16x2_bits(p2 - bf16_bits_to_f32(h23 & 0xFFFFu), p3 - bf16_bits_to_f32(h23 >> 16));
            const uint32_t pb[2] = {movmatrix_trans(h01), movmatrix_trans(h23)};
            const uint32_t pl[2] = {movmatrix_trans(l01), movmatrix_trans(l23)};
            // ---- O^T[HD x 8] += V^T P^T ----
            {
                const int key = warp * 16 + ((j >> 1) << 3) + rr;
#pragma unroll
                for (int mi = 0; mi < HD / 16; ++mi) {
                    uint32_t a[4];
                    ldmatrix_x4_trans(a, tile_addr<C>(vb, key, mi * 16 + ((j & 1) << 3)));
                    mma_bf16_16816(o[mi], a, pb, o[mi]);
                    mma_bf16_16816(o[mi], a, pl, o[mi]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // per-head l over the 8 lanes g of each tq
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, off);
            l1 += __shfl_xor_sync(0xffffffffu, l1, off);
        }
    }
    __syncthreads();  // all TMA traffic has landed and been consumed: reuse the stages

    // ---- merge the consumer warps in shared memory ----
    float* osm = reinterpret_cast<float*>(smem);                  // [WARPS][8][HD]
    float* msm = osm + C::WARPS * 8 * HD;                         // [WARPS][8]
    float* lsm = msm + C::WARPS * 8;                              // [WARPS][8]
    if (warp < C::WARPS) {
        float* ow = osm + warp * 8 * HD;
#pragma unroll
        for (int i = 0; i < HD / 16; ++i) {
            const int d = i * 16 + g;
            ow[(2 * tq) * HD + d] = o[i][0];
            ow[(2 * tq + 1) * HD + d] = o[i][1];
            ow[(2 * tq) * HD + d + 8] = o[i][2];
            ow[(2 * tq + 1) * HD + d + 8] = o[i][3];
        }
        if (g == 0) {
            msm[warp * 8 + 2 * tq] = m0;
            msm[warp * 8 + 2 * tq + 1] = m1;
            lsm[warp * 8 + 2 * tq] = l0;
            lsm[warp * 8 + 2 * tq + 1] = l1;
        }
    }
    __syncthreads();
    const int nh = p.heads;
    for (int idx = threadIdx.x; idx < nh * HD; idx += blockDim.x) {
        const int h = idx / HD, d = idx - h * HD;
        float m = -INFINITY;
#pragma unroll
        for (int w = 0; w < C::WARPS; ++w) m = fmaxf(m, msm[w * 8 + h]);
        const float mu = m == -INFINITY ? 0.f : m;
        float l = 0.f, acc = 0.f;
#pragma unroll
        for (int w = 0; w < C::WARPS; ++w) {
            const float f = exp2f(msm[w * 8 + h] - mu);
            l += f * lsm[w * 8 + h];
            acc += f * osm[(w * 8 + h) * HD + d];
        }
        if (p.nsplit == 1) {
            p.out[((size_t)r * nh + h) * HD + d] = (uint16_t)f32_to_bf16_bits(acc / l);
        } else {
            const size_t pi = ((size_t)r * p.nsplit + split) * 8 + h;
            p.part_o[pi * HD + d] = acc;
            if (d == 0) p.part_ml[pi] = make_float2(m, l);
        }
    }
}

// Merges the split-KV partials (log-sum-exp weights).  One CTA per (row, head), one
// thread per output column.  The per-split (m, l) pairs are read once, in parallel,
// into shared memory; the column loop then issues its loads independently.
constexpr int kMaxSplits = 1024;

template <int HD>
__global__ void __launch_bounds__(HD) attn_combine_kernel(const float* __restrict__ part_o,
                                                          const float2* __restrict__ part_ml, int nsplit,
                                                          int heads, uint16_t* __restrict__ out) {
    __shared__ float s_w[kMaxSplits];
    __shared__ float s_red[HD / 32];
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x / heads, h = blockIdx.x - r * heads, d = threadIdx.x;
    const float2* ml = part_ml + (size_t)r * nsplit * 8 + h;
    float mloc = -INFINITY;
    for (int s = d; s < nsplit; s += HD) {
        const float m = __ldg(&ml[(size_t)s * 8].x);
        s_w[s] = m;
        mloc = fmaxf(mloc, m);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, off));
    if ((d & 31) == 0) s_red[d >> 5] = mloc;
    __syncthreads();
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < HD / 32; ++i) m = fmaxf(m, s_red[i]);
    const float mu = m == -INFINITY ? 0.f : m;
    __syncthreads();
    float lloc = 0.f;
    for (int s = d; s < nsplit; s += HD) {
        const float f = exp2f(s_w[s] - mu);
        lloc += f * __ldg(&ml[(size_t)s * 8].y);
        s_w[s] = f;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) lloc += __shfl_xor_sync(0xffffffffu, lloc, off);
    if ((d & 31) == 0) s_red[d >> 5] = lloc;
    __syncthreads();
    float l = 0.f;
#pragma unroll
    for (int i = 0; i < HD / 32; ++i) l += s_red[i];
    const float* po = part_o + ((size_t)r * nsplit * 8 + h) * HD + d;
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
    int s = 0;
    for (; s + 4 <= nsplit; s += 4) {
        acc0 += s_w[s] * __ldg(po + (size_t)s * 8 * HD);
        acc1 += s_w[s + 1] * __ldg(po + (size_t)(s + 1) * 8 * HD);
        acc2 += s_w[s + 2] * __ldg(po + (size_t)(s + 2) * 8 * HD);
        acc3 += s_w[s + 3] * __ldg(po + (size_t)(s + 3) * 8 * HD);
    }
    for (; s < nsplit; ++s) acc0 += s_w[s] * __ldg(po + (size_t)s * 8 * HD);
    out[((size_t)r * heads + h) * HD + d] = (uint16_t)f32_to_bf16_bits(((acc0 + acc1) + (acc2 + acc3)) / l);
}

// Appends rows to the bf16 cache, rounding f32 input to nearest even.
__global__ void kv_append_f32_kernel(const float* __restrict__ k, const float* __restrict__ v,
                                     uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, long long n) {
    pdl_trigger();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    kc[i] = (uint16_t)f32_to_bf16_bits(k[i]);
    vc[i] = (uint16_t)f32_to_bf16_bits(v[i]);
}

// KVCache.append into a ring cache: row i of k/v (f32 or bf16) is position start + i, slot
// (start + i) % ring, also written to row ring + slot when slot < mirror.  Only the last
// `ring` rows are written (earlier ones would be overwritten by later rows of the call).
__global__ void kv_append_ring_kernel(const void* __restrict__ k, const void* __restrict__ v, int src_f32, int rows,
                                      int start, int hd, int ring, int mirror, uint16_t* __restrict__ kc,
                                      uint16_t* __restrict__ vc) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int first = rows > ring ? rows - ring : 0;
    if (i >= (long long)(rows - first) * hd) return;
    const int r = first + (int)(i / hd), d = (int)(i % hd);
    const size_t src = (size_t)r * hd + d;
    const uint16_t kb = src_f32 ? (uint16_t)f32_to_bf16_bits(static_cast<const float*>(k)[src])
                                : static_cast<const uint16_t*>(k)[src];
    const uint16_t vb = src_f32 ? (uint16_t)f32_to_bf16_bits(static_cast<const float*>(v)[src])
                                : static_cast<const uint16_t*>(v)[src];
    const int slot = (start + r) % ring;
    kc[(size_t)slot * hd + d] = kb;
    vc[(size_t)slot * hd + d] = vb;
    if (slot < mirror) {
        kc[(size_t)(ring + slot) * hd + d] = kb;
        vc[(size_t)(ring + slot) * hd + d] = vb;
    }
}

template <int HD, bool kNarrow>
g4_status launch_attn_t(g4_ctx* ctx, const CUtensorMap& km, const CUtensorMap& vm, const uint16_t* q,
                        int rows, int heads, int keylen, int qpos0, int sliding, int window, uint16_t* out,
                        int kv_row0, void* fixed_scratch, size_t fixed_bytes, const g4_rows* map, int seq_stride,
                        int ring) {
    using C = AttnCfg<HD, kNarrow>;
    // Longest key range of any row decides the split.  With device-side positions the
    // host does not know the lengths: plan for a full sequence (or a full window).
    int lmax;
    if (map) {
        lmax = sliding ? min(window, seq_stride) : seq_stride;
    } else {
        const int qp_last = qpos0 + rows - 1;
        lmax = min(qp_last, keylen - 1) + 1;
        if (sliding) lmax = min(lmax, window);
    }
    const int ntiles = (lmax + C::KT - 1) / C::KT;
    int nsplit = (2 * ctx->num_sms + rows - 1) / rows;
    nsplit = min(nsplit, max(1, (ntiles + 1) / 2));
    // Batched rows: split a row's keys only as far as needed to give every SM a CTA, and
    // not at all from a third of the SM count up: there one CTA per row streams the whole
    // key range (HBM-bound) and the combine pass, a link more in the decode chain, costs
    // more than the idle SMs (measured at 64 and 128 rows; at 32 rows the split wins).
    if (map)
        nsplit = rows * 3 > ctx->num_sms ? 1 : max(1, min((ctx->num_sms + rows - 1) / rows, (ntiles + 1) / 2));
    nsplit = max(nsplit, 1);
    const int tiles_per_split = (ntiles + nsplit - 1) / nsplit;
    nsplit = (ntiles + tiles_per_split - 1) / tiles_per_split;
    if (nsplit < 1) nsplit = 1;
    if (nsplit > kMaxSplits) return g4::set_error(G4_ERR_UNSUPPORTED, "attention: %d key splits", nsplit);

    AttnParams p{};
    p.q = q;
    p.out = out;
    p.err = ctx->d_err;
    p.heads = heads;
    p.keylen = keylen;
    p.qpos0 = qpos0;
    p.sliding = sliding;
    p.window = window;
    p.ring = ring;
    p.nsplit = nsplit;
    p.split_keys = tiles_per_split * C::KT;
    p.kv_row0 = kv_row0;
    if (map) {
        p.seq_pos = map->seq_pos;
        p.seq_base = map->seq_base;
        p.rows_per_seq = map->rows_per_seq;
        p.pos0 = map->pos0;
        p.seq_stride = seq_stride;
        p.history_ready = (map->flags & G4_ROWS_HISTORY_READY) ? 1 : 0;
    }
    if (nsplit > 1) {
        const size_t ob = (size_t)rows * nsplit * 8 * HD * sizeof(float);
        const size_t mb = (size_t)rows * nsplit * 8 * sizeof(float2);
        void* scratch = fixed_scratch;
        if (scratch) {
            if (ob + mb + 256 > fixed_bytes)
                return g4::set_error(G4_ERR_RANGE,
                                     "attention: %d rows x %d key splits need %zu bytes of scratch; the static "
                                     "scratch of g4_attention_noalloc holds %zu bytes",
                                     rows, nsplit, ob + mb + 256, fixed_bytes);
        } else {
            g4_status st = g4::ensure_workspace(ctx, ob + mb + 256);
            if (st) return st;
            scratch = ctx->ws;
        }
        p.part_o = static_cast<float*>(scratch);
        p.part_ml = reinterpret_cast<float2*>(static_cast<uint8_t*>(scratch) + ((ob + 255) & ~size_t(255)));
    }
    static std::atomic<uint64_t> attr_set{0};
    if (!(attr_set.load() & (1ull << ctx->device))) {
        G4_CHECK_CUDA(cudaFuncSetAttribute(attn_decode_kernel<HD, kNarrow>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           C::SMEM));
        attr_set.fetch_or(1ull << ctx->device);
    }
    g4_status st = g4::launch(ctx, "attn_decode_kernel", attn_decode_kernel<HD, kNarrow>, dim3(nsplit, rows), dim3(C::THREADS),
                              C::SMEM, 1, km, vm, p);
    if (st) return st;
    if (nsplit > 1)
        return g4::launch(ctx, "attn_combine_kernel", attn_combine_kernel<HD>, dim3(rows * heads), dim3(HD), 0, 1,
                          static_cast<const float*>(p.part_o), static_cast<const float2*>(p.part_ml), nsplit, heads,
                          out);
    return G4_OK;
}

}  // namespace

namespace g4 {

g4_status make_kv_maps(g4_kv* kv) {
    CUtensorMap* maps[4] = {&kv->kmap, &kv->vmap, &kv->kmap_narrow, &kv->vmap_narrow};
    for (int i = 0; i < 4; ++i) {
        const uint32_t kt = (i < 2 ? 16384u : 8192u) / (uint32_t)kv->hd;
        g4_status st = encode_tensor_map_2d(maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (i & 1) ? kv->v : kv->k,
                                            kv->hd, kv->rows_total, (uint64_t)kv->hd * 2, 64, kt,
                                            CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
    }
    return G4_OK;
}

template <int HD>
g4_status launch_attn_hd(g4_ctx* ctx, const g4_kv* kv, int kv_row0, const uint16_t* q, int rows, int heads,
                         int keylen, int qpos0, int sliding, int window, uint16_t* out, void* fixed_scratch,
                         size_t fixed_bytes, const g4_rows* map, int seq_stride) {
    // Batched decode of sliding layers with more rows than SMs: one CTA per row's short
    // window, two per SM, so the whole grid is resident at once.  (Global layers stream
    // long key ranges, where the wide tiles measured faster.)
    if (map && sliding && rows > ctx->num_sms)
        return launch_attn_t<HD, true>(ctx, kv->kmap_narrow, kv->vmap_narrow, q, rows, heads, keylen, qpos0, sliding,
                                       window, out, kv_row0, fixed_scratch, fixed_bytes, map, seq_stride, kv->ring);
    return launch_attn_t<HD, false>(ctx, kv->kmap, kv->vmap, q, rows, heads, keylen, qpos0, sliding, window, out,
                                    kv_row0, fixed_scratch, fixed_bytes, map, seq_stride, kv->ring);
}

g4_status launch_attention(g4_ctx* ctx, const g4_kv* kv, int kv_row0, const uint16_t* q, int rows, int heads,
                           int keylen, int qpos0, int sliding, int window, uint16_t* out, void* fixed_scratch,
                           size_t fixed_bytes, const g4_rows* map, int seq_stride) {
    switch (kv->hd) {
        case 64: return launch_attn_hd<64>(ctx, kv, kv_row0, q, rows, heads, keylen, qpos0, sliding, window, out, fixed_scratch, fixed_bytes, map, seq_stride);
        case 128: return launch_attn_hd<128>(ctx, kv, kv_row0, q, rows, heads, keylen, qpos0, sliding, window, out, fixed_scratch, fixed_bytes, map, seq_stride);
        case 256: return launch_attn_hd<256>(ctx, kv, kv_row0, q, rows, heads, keylen, qpos0, sliding, window, out, fixed_scratch, fixed_bytes, map, seq_stride);
        case 512: return launch_attn_hd<512>(ctx, kv, kv_row0, q, rows, heads, keylen, qpos0, sliding, window, out, fixed_scratch, fixed_bytes, map, seq_stride);
        default: return set_error(G4_ERR_UNSUPPORTED, "attention: head dim %d (64/128/256/512 supported)", kv->hd);
    }
}

}  // namespace g4

extern "C" {

g4_status g4_kv_create(g4_ctx* ctx, int hd, int capacity, g4_kv** out) {
    if (!out) return g4::set_error(G4_ERR_INVALID, "g4_kv_create: null out");
    *out = nullptr;
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (hd != 64 && hd != 128 && hd != 256 && hd != 512)
        return g4::set_error(G4_ERR_UNSUPPORTED, "g4_kv_create: head dim %d (64/128/256/512 supported)", hd);
    if (capacity <= 0) return g4::set_error(G4_ERR_INVALID, "g4_kv_create: capacity %d", capacity);
    g4_kv* kv = new g4_kv();
    kv->ctx = ctx;
    kv->hd = hd;
    kv->capacity = capacity;
    kv->rows_total = capacity;
    const size_t bytes = (size_t)capacity * hd * 2;
    cudaError_t e = cudaMalloc(&kv->k, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&kv->v, bytes);
    // Zero-fill: masked keys must hold finite values (p = 0 times V must stay 0).
    if (e == cudaSuccess) e = cudaMemsetAsync(kv->k, 0, bytes, ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(kv->v, 0, bytes, ctx->stream);
    if (e != cudaSuccess) {
        g4_kv_destroy(kv);
        return g4::cuda_error(e, "g4_kv_create");
    }
    st = g4::make_kv_maps(kv);
    if (st) {
        g4_kv_destroy(kv);
        return st;
    }
    *out = kv;
    return G4_OK;
}

g4_status g4_kv_create_ring(g4_ctx* ctx, int hd, int capacity, int ring, int nseq, g4_kv** out) {
    if (!out) return g4::set_error(G4_ERR_INVALID, "g4_kv_create_ring: null out");
    *out = nullptr;
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (hd != 64 && hd != 128 && hd != 256 && hd != 512)
        return g4::set_error(G4_ERR_UNSUPPORTED, "g4_kv_create_ring: head dim %d (64/128/256/512 supported)", hd);
    const int mirror = 16384 / hd;
    if (capacity <= 0 || nseq <= 0) return g4::set_error(G4_ERR_INVALID, "g4_kv_create_ring: capacity %d, %d sequences",
                                                         capacity, nseq);
    if (ring < mirror)
        return g4::set_error(G4_ERR_INVALID, "g4_kv_create_ring: ring of %d slots (at least %d at head dim %d)", ring,
                             mirror, hd);
    if ((long long)nseq * (ring + mirror) > 0x7fffffffLL)
        return g4::set_error(G4_ERR_RANGE, "g4_kv_create_ring: %d sequences x %d rows", nseq, ring + mirror);
    g4_kv* kv = new g4_kv();
    kv->ctx = ctx;
    kv->hd = hd;
    kv->capacity = capacity;
    kv->ring = ring;
    kv->mirror = mirror;
    kv->nseq = nseq;
    kv->seq_rows = ring + mirror;
    kv->rows_total = nseq * kv->seq_rows;
    const size_t bytes = (size_t)kv->rows_total * hd * 2;
    cudaError_t e = cudaMalloc(&kv->k, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&kv->v, bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(kv->k, 0, bytes, ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(kv->v, 0, bytes, ctx->stream);
    if (e != cudaSuccess) {
        g4_kv_destroy(kv);
        return g4::cuda_error(e, "g4_kv_create_ring");
    }
    st = g4::make_kv_maps(kv);
    if (st) {
        g4_kv_destroy(kv);
        return st;
    }
    *out = kv;
    return G4_OK;
}

g4_status g4_kv_layout(const g4_kv* kv, int* ring, int* seq_rows, int* nseq) {
    if (!kv) return g4::set_error(G4_ERR_INVALID, "null kv");
    if (ring) *ring = kv->ring;
    if (seq_rows) *seq_rows = kv->ring ? kv->seq_rows : kv->rows_total;
    if (nseq) *nseq = kv->nseq;
    return G4_OK;
}

g4_status g4_kv_destroy(g4_kv* kv) {
    if (!kv) return G4_OK;
    if (kv->ctx) {
        cudaSetDevice(kv->ctx->device);
        cudaStreamSynchronize(kv->ctx->stream);
    }
    cudaFree(kv->k);
    cudaFree(kv->v);
    delete kv;
    return G4_OK;
}

g4_status g4_kv_append(g4_ctx* ctx, g4_kv* kv, const void* k, const void* v, int rows, int start_pos,
                       g4_dtype src_dtype) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!kv || !k || !v) return g4::set_error(G4_ERR_INVALID, "g4_kv_append: null argument");
    // gemma4-webgpu.js:129-130
    if (start_pos != kv->length)
        return g4::set_error(G4_ERR_INVALID, "KV append position %d != cache length %d", start_pos, kv->length);
    if (rows < 0 || start_pos + rows > kv->capacity)
        return g4::set_error(G4_ERR_RANGE, "KV cache capacity %d exceeded", kv->capacity);
    if (rows == 0) return G4_OK;
    if (kv->ring) {
        if (kv->nseq != 1)
            return g4::set_error(G4_ERR_INVALID, "g4_kv_append: ring cache of %d sequences (append K/V with "
                                 "g4_qkv_post_kv)", kv->nseq);
        if (src_dtype != G4_BF16 && src_dtype != G4_F32)
            return g4::set_error(G4_ERR_INVALID, "g4_kv_append: dtype %d", (int)src_dtype);
        const long long n = (long long)std::min(rows, kv->ring) * kv->hd;
        st = g4::launch(ctx, "kv_append_ring_kernel", kv_append_ring_kernel, dim3((unsigned)((n + 255) / 256)),
                        dim3(256), 0, 1, k, v, src_dtype == G4_F32 ? 1 : 0, rows, start_pos, kv->hd, kv->ring,
                        kv->mirror, kv->k, kv->v);
        if (st) return st;
        kv->length += rows;
        return G4_OK;
    }
    const size_t n = (size_t)rows * kv->hd;
    uint16_t* kd = kv->k + (size_t)start_pos * kv->hd;
    uint16_t* vd = kv->v + (size_t)start_pos * kv->hd;
    if (src_dtype == G4_BF16) {
        G4_CHECK_CUDA(cudaMemcpyAsync(kd, k, n * 2, cudaMemcpyDeviceToDevice, ctx->stream));
        G4_CHECK_CUDA(cudaMemcpyAsync(vd, v, n * 2, cudaMemcpyDeviceToDevice, ctx->stream));
    } else if (src_dtype == G4_F32) {
        st = g4::launch(ctx, "kv_append_f32_kernel", kv_append_f32_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256),
                        0, 1, static_cast<const float*>(k), static_cast<const float*>(v), kd, vd, (long long)n);
        if (st) return st;
    } else {
        return g4::set_error(G4_ERR_INVALID, "g4_kv_append: dtype %d", (int)src_dtype);
    }
    kv->length += rows;
    return G4_OK;
}

g4_status g4_kv_info(const g4_kv* kv, int* length, int* hd, int* capacity) {
    if (!kv) return g4::set_error(G4_ERR_INVALID, "null kv");
    if (length) *length = kv->length;
    if (hd) *hd = kv->hd;
    if (capacity) *capacity = kv->capacity;
    return G4_OK;
}

g4_status g4_kv_reset(g4_kv* kv) {
    if (!kv) return g4::set_error(G4_ERR_INVALID, "null kv");
    kv->length = 0;
    return G4_OK;
}

g4_status g4_kv_buffers(const g4_kv* kv, void** k, void** v) {
    if (!kv) return g4::set_error(G4_ERR_INVALID, "null kv");
    if (k) *k = kv->k;
    if (v) *v = kv->v;
    return G4_OK;
}

}  // extern "C"

namespace g4 {

g4_status check_ring(const char* name, const g4_kv* kv, int sliding, int window, int span);

// The argument rules of GPUOps.attention with host-side positions, shared by g4_attention
// and g4_attention_noalloc (`name` prefixes the messages).  *empty is set when rows == 0.
g4_status check_attention_args(const char* name, g4_ctx* ctx, const void* q_bf16, const g4_kv* kv, int rows,
                               int heads, int hd, int keylen, int qpos0, int sliding, int window, const void* out_bf16,
                               bool* empty) {
    *empty = false;
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!kv || !q_bf16 || !out_bf16) return g4::set_error(G4_ERR_INVALID, "%s: null argument", name);
    if (rows < 0) return g4::set_error(G4_ERR_INVALID, "%s: rows %d", name, rows);
    if (rows == 0) {
        *empty = true;
        return G4_OK;
    }
    if (hd != kv->hd) return g4::set_error(G4_ERR_INVALID, "%s: hd %d != cache hd %d", name, hd, kv->hd);
    if (heads < 1 || heads > 8)
        return g4::set_error(G4_ERR_UNSUPPORTED, "%s: %d heads per KV head (1..8 supported)", name, heads);
    if (keylen < 1 || keylen > kv->length)
        return g4::set_error(G4_ERR_INVALID, "%s: keylen %d outside cache length %d", name, keylen, kv->length);
    if (qpos0 < 0 || qpos0 + rows > keylen)
        return g4::set_error(G4_ERR_INVALID, "%s: query positions [%d,%d) not below keylen %d", name, qpos0,
                             qpos0 + rows, keylen);
    if (sliding && window < 1) return g4::set_error(G4_ERR_INVALID, "%s: window %d", name, window);
    if (reinterpret_cast<uintptr_t>(q_bf16) % 16 != 0)
        return g4::set_error(G4_ERR_INVALID, "%s: q must be 16-byte aligned", name);
    return check_ring(name, kv, sliding, window, keylen - qpos0);
}

// A ring cache holds the last `ring` positions of each sequence: it serves sliding-window
// attention whose queries, with `span` = keylen - first query position, never reach back
// further than that (span + window - 1 <= ring).
g4_status check_ring(const char* name, const g4_kv* kv, int sliding, int window, int span) {
    if (!kv->ring) return G4_OK;
    if (!sliding)
        return g4::set_error(G4_ERR_INVALID, "%s: a ring KV cache (%d slots) serves sliding-window attention only",
                             name, kv->ring);
    if ((long long)span + window - 1 > kv->ring)
        return g4::set_error(G4_ERR_RANGE,
                             "%s: %d query positions with a window of %d need %lld ring slots; the cache has %d",
                             name, span, window, (long long)span + window - 1, kv->ring);
    return G4_OK;
}

}  // namespace g4

extern "C" {

g4_status g4_attention(g4_ctx* ctx, const void* q_bf16, const g4_kv* kv, int rows, int heads, int hd,
                       int keylen, int qpos0, int sliding, int window, void* out_bf16) {
    bool empty = false;
    g4_status st = g4::check_attention_args("g4_attention", ctx, q_bf16, kv, rows, heads, hd, keylen, qpos0, sliding,
                                            window, out_bf16, &empty);
    if (st || empty) return st;
    return g4::launch_attention(ctx, kv, 0, static_cast<const uint16_t*>(q_bf16), rows, heads, keylen, qpos0,
                                sliding ? 1 : 0, window, static_cast<uint16_t*>(out_bf16));
}


g4_status g4_attention_rows(g4_ctx* ctx, const void* q_bf16, const g4_kv* kv, int rows, int heads, int hd,
                            const g4_rows* map, int seq_stride, int sliding, int window, void* out_bf16) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!kv || !q_bf16 || !out_bf16 || !map || !map->seq_pos || map->rows_per_seq < 1)
        return g4::set_error(G4_ERR_INVALID, "g4_attention_rows: null argument");
    if (rows < 0) return g4::set_error(G4_ERR_INVALID, "g4_attention_rows: rows %d", rows);
    if (rows == 0) return G4_OK;
    if (hd != kv->hd) return g4::set_error(G4_ERR_INVALID, "g4_attention_rows: hd %d != cache hd %d", hd, kv->hd);
    if (heads < 1 || heads > 8)
        return g4::set_error(G4_ERR_UNSUPPORTED, "g4_attention_rows: %d heads per KV head (1..8 supported)", heads);
    if (seq_stride < 1 || (long long)(map->seq_base + (rows - 1) / map->rows_per_seq + 1) * seq_stride > kv->rows_total)
        return g4::set_error(G4_ERR_RANGE, "g4_attention_rows: sequences beyond the cache (%d rows)", kv->rows_total);
    if (sliding && window < 1) return g4::set_error(G4_ERR_INVALID, "g4_attention_rows: window %d", window);
    if (kv->ring && seq_stride != kv->seq_rows)
        return g4::set_error(G4_ERR_INVALID, "g4_attention_rows: seq_stride %d of a ring cache must be its %d rows per "
                             "sequence", seq_stride, kv->seq_rows);
    st = g4::check_ring("g4_attention_rows", kv, sliding, window, map->rows_per_seq);
    if (st) return st;
    return g4::launch_attention(ctx, kv, 0, static_cast<const uint16_t*>(q_bf16), rows, heads, 0, 0, sliding ? 1 : 0,
                                window, static_cast<uint16_t*>(out_bf16), nullptr, 0, map, seq_stride);
}

}  // extern "C"

// ------------------------------------------------ attention without allocation --
//
// Some callers cannot let a library call cudaMalloc: hosts that hand every byte of
// device memory to their own pool at start-up (as a WebGPU-style runtime does), and
// serving loops where cudaMalloc's implicit device-wide synchronisation would stall
// the other streams.  g4_attention grows a context workspace with cudaMalloc when a
// long key range is split across CTAs; g4_attention_noalloc instead keeps the split
// partials in the fixed array below, which every GPU that loads this library holds
// (8 MiB) until the process exits.

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
__device__ __align__(256) uint8_t g_attn_noalloc_scratch[kNoAllocScratchBytes];

// In host code g_attn_noalloc_scratch names a host-side shadow, not device memory, so
// its device address is looked up once per device (with that device current) and cached.
g4_status noalloc_scratch(int device, void** out) {
    static std::mutex mu;
    static void* ptrs[64] = {};
    if (device < 0 || device >= 64) return g4::set_error(G4_ERR_INVALID, "g4_attention_noalloc: device %d", device);
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
        if (e != cudaSuccess) return g4::cuda_error(e, "g4_attention_noalloc: cudaGetSymbolAddress");
        ptrs[device] = p;
    }
    *out = ptrs[device];
    return G4_OK;
}

}  // namespace

extern "C" g4_status g4_attention_noalloc(g4_ctx* ctx, const void* q_bf16, const g4_kv* kv, int rows, int heads,
                                          int hd, int keylen, int qpos0, int sliding, int window, void* out_bf16) {
    bool empty = false;
    g4_status st = g4::check_attention_args("g4_attention_noalloc", ctx, q_bf16, kv, rows, heads, hd, keylen, qpos0,
                                            sliding, window, out_bf16, &empty);
    if (st || empty) return st;
    void* scratch = nullptr;
    st = noalloc_scratch(ctx->device, &scratch);
    if (st) return st;
    return g4::launch_attention(ctx, kv, 0, static_cast<const uint16_t*>(q_bf16), rows, heads, keylen, qpos0,
                                sliding ? 1 : 0, window, static_cast<uint16_t*>(out_bf16), scratch,
                                kNoAllocScratchBytes);
}
