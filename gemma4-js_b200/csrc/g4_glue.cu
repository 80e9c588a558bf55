// g4_glue.cu -- the row-wise operators of the reference runtime around the W4A16 path,
// fused where the model graph chains them.
//
// Reference shaders (custom-webgpu/gpu-runtime.js): RMS_SHADER :1104-1118, ADD_SCALE
// :1120-1128, SCALE :1130-1137, GELU_MUL :1139-1157, GELU_PLE :1159-1173, NORM_ROPE
// :1175-1202, PLE_MIX :1250-1263, BF16_HEAD :1265-1277 and topK :1396-1425.  Each
// kernel keeps the shader's f32 arithmetic; activations that feed a W4A16 linear or
// the attention are emitted in bf16 (round to nearest even).
//
// Positions: rows of a batch map to sequences through (seq_base, rows_per_seq):
// row r belongs to sequence seq_base + r / rows_per_seq at offset r % rows_per_seq,
// and its absolute position is seq_pos[seq] + offset.  seq_pos lives on the device,
// so a captured decode step replays correctly as positions advance.
#include <stdio.h>

#include "g4_attention.cuh"
#include "g4_common.cuh"
#include "g4_glue.cuh"

namespace {

using namespace g4dev;

constexpr int kRowThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float s = 0.f;
    const int nw = blockDim.x >> 5;
    for (int i = 0; i < nw; ++i) s += red[i];
    return s;
}

__device__ __forceinline__ int row_position(const G4Rows& R, int r) {
    const int seq = R.seq_base + r / R.rows_per_seq;
    return (R.seq_pos ? R.seq_pos[seq] : 0) + R.pos0 + r % R.rows_per_seq;
}
__device__ __forceinline__ int row_seq(const G4Rows& R, int r) { return R.seq_base + r / R.rows_per_seq; }

// A linear's output as partial planes (g4_planes): the slices are added in order, the
// same bits the linear's own last pass (splitk_sum_kernel) produces.
struct Planes {
    const float* base;
    long long stride;
    int count, ld;
};
// The planes are summed in slice order (a = p0; a += p1; ...), the order of the
// splitk_sum pass; the loads of up to 8 slices are issued before their adds, so a
// thread waits for one L2 round trip per 8 slices instead of one per slice.
constexpr int kPlaneBatch = 8;
__device__ __forceinline__ float ld_planes(const Planes& P, size_t off) {
    const float* p = P.base + off;
    float a = __ldg(p);
    for (int s0 = 1; s0 < P.count; s0 += kPlaneBatch) {
        float b[kPlaneBatch];
#pragma unroll
        for (int j = 0; j < kPlaneBatch; ++j) b[j] = s0 + j < P.count ? __ldg(p + (size_t)(s0 + j) * P.stride) : 0.f;
#pragma unroll
        for (int j = 0; j < kPlaneBatch; ++j)
            if (s0 + j < P.count) a += b[j];
    }
    return a;
}
__device__ __forceinline__ float4 ld4_planes(const Planes& P, size_t off) {
    const float* p = P.base + off;
    float4 a = __ldg(reinterpret_cast<const float4*>(p));
    for (int s0 = 1; s0 < P.count; s0 += kPlaneBatch) {
        float4 b[kPlaneBatch];
#pragma unroll
        for (int j = 0; j < kPlaneBatch; ++j)
            b[j] = s0 + j < P.count ? __ldg(reinterpret_cast<const float4*>(p + (size_t)(s0 + j) * P.stride))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < kPlaneBatch; ++j) {
            if (s0 + j < P.count) {
                a.x += b[j].x;
                a.y += b[j].y;
                a.z += b[j].z;
                a.w += b[j].w;
            }
        }
    }
    return a;
}

// ld4_planes at two offsets, every load of both issued before the first add (a warp issues
// in order, so an add that waits on a load holds back the loads behind it).
__device__ __forceinline__ void ld4_planes2(const Planes& P, size_t off_a, size_t off_b, float4& a, float4& b) {
    const float* pa = P.base + off_a;
    const float* pb = P.base + off_b;
    a = __ldg(reinterpret_cast<const float4*>(pa));
    b = __ldg(reinterpret_cast<const float4*>(pb));
    for (int s0 = 1; s0 < P.count; s0 += kPlaneBatch / 2) {
        float4 ba[kPlaneBatch / 2], bb[kPlaneBatch / 2];
#pragma unroll
        for (int j = 0; j < kPlaneBatch / 2; ++j) {
            const bool in = s0 + j < P.count;
            const size_t o = (size_t)(s0 + j) * P.stride;
            ba[j] = in ? __ldg(reinterpret_cast<const float4*>(pa + o)) : make_float4(0.f, 0.f, 0.f, 0.f);
            bb[j] = in ? __ldg(reinterpret_cast<const float4*>(pb + o)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < kPlaneBatch / 2; ++j) {
            if (s0 + j < P.count) {
                a.x += ba[j].x; a.y += ba[j].y; a.z += ba[j].z; a.w += ba[j].w;
                b.x += bb[j].x; b.y += bb[j].y; b.z += bb[j].z; b.w += bb[j].w;
            }
        }
    }
}

// RMS_SHADER: y = x * rsqrt(mean(x^2) + eps) * scale (scale optional).
__global__ void __launch_bounds__(kRowThreads) rms_kernel(const float* __restrict__ x, const float* __restrict__ scale,
                                                          int width, float eps, void* __restrict__ out, int out_bf16) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    const int r = blockIdx.x;
    const float* xr = x + (size_t)r * width;
    float ss = 0.f;
    for (int i = threadIdx.x; i < width; i += blockDim.x) ss += xr[i] * xr[i];
    const float inv = rsqrtf(block_sum(ss, red) / (float)width + eps);
    for (int i = threadIdx.x; i < width; i += blockDim.x) {
        const float v = xr[i] * inv * (scale ? scale[i] : 1.f);
        if (out_bf16)
            reinterpret_cast<uint16_t*>(out)[(size_t)r * width + i] = (uint16_t)f32_to_bf16_bits(v);
        else
            reinterpret_cast<float*>(out)[(size_t)r * width + i] = v;
    }
}

// RMS_SHADER for width % 4 == 0, width <= 4096: one float4 of the row per thread, loaded
// once (the scale, immutable, before the PDL wait), one reduction.
__global__ void __launch_bounds__(1024) rms4_kernel(const float* __restrict__ x, const float* __restrict__ scale,
                                                    int width, float eps, void* __restrict__ out, int out_bf16) {
    pdl_trigger();
    __shared__ float red[32];
    const int r = blockIdx.x, i = threadIdx.x * 4;
    const bool on = i < width;
    float4 sc = make_float4(1.f, 1.f, 1.f, 1.f), v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (on && scale) sc = __ldg(reinterpret_cast<const float4*>(scale + i));
    pdl_wait();
    if (on) v = *reinterpret_cast<const float4*>(x + (size_t)r * width + i);
    const float inv = rsqrtf(block_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w, red) / (float)width + eps);
    if (!on) return;
    const float4 o = make_float4(v.x * inv * sc.x, v.y * inv * sc.y, v.z * inv * sc.z, v.w * inv * sc.w);
    if (out_bf16)
        *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(out) + (size_t)r * width + i) =
            make_uint2(pack_bf16x2_bits(o.x, o.y), pack_bf16x2_bits(o.z, o.w));
    else
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)r * width + i) = o;
}

// ADD_SCALE: y = (a + b) * s.
__global__ void add_scale_kernel(const float* __restrict__ a, const float* __restrict__ b, long long n, float s,
                                 float* __restrict__ y) {
    pdl_trigger();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = (a[i] + b[i]) * s;
}

// RMS_SHADER + ADD_SCALE (+ the next RMS_SHADER) of one residual update:
//   h = (h + rms(y) * w_post) * skip;  x = bf16(w_next ? rms(h) * w_next : h)
// One CTA per row, one float4 of the row per thread, kept in registers across the
// two reductions (width % 4 == 0, width <= 4096).
__global__ void __launch_bounds__(1024) post_norm_add_kernel(float* __restrict__ h, Planes y,
                                                             const float* __restrict__ w_post, float skip,
                                                             const float* __restrict__ w_next, int width, float eps,
                                                             uint16_t* __restrict__ x_out) {
    pdl_trigger();
    __shared__ float red[32];
    const int r = blockIdx.x, i = threadIdx.x * 4;
    const bool on = i < width;
    float4 yv = make_float4(0.f, 0.f, 0.f, 0.f), hv = yv, wp = yv, wn = yv;
    if (on) {  // the norm weights are immutable: fetched while the predecessor drains
        wp = __ldg(reinterpret_cast<const float4*>(w_post + i));
        if (w_next) wn = __ldg(reinterpret_cast<const float4*>(w_next + i));
    }
    pdl_wait();
    if (on) {  // h first: its load is in flight with the planes' (one L2 round trip in all)
        hv = *reinterpret_cast<const float4*>(h + (size_t)r * width + i);
        yv = ld4_planes(y, (size_t)r * y.ld + i);
    }
    const float inv = rsqrtf(block_sum(yv.x * yv.x + yv.y * yv.y + yv.z * yv.z + yv.w * yv.w, red) / (float)width + eps);
    hv.x = (hv.x + yv.x * inv * wp.x) * skip;
    hv.y = (hv.y + yv.y * inv * wp.y) * skip;
    hv.z = (hv.z + yv.z * inv * wp.z) * skip;
    hv.w = (hv.w + yv.w * inv * wp.w) * skip;
    if (on) *reinterpret_cast<float4*>(h + (size_t)r * width + i) = hv;
    if (!x_out) return;
    float4 o = hv;
    if (w_next) {
        const float inv2 =
            rsqrtf(block_sum(hv.x * hv.x + hv.y * hv.y + hv.z * hv.z + hv.w * hv.w, red) / (float)width + eps);
        if (on) o = make_float4(hv.x * inv2 * wn.x, hv.y * inv2 * wn.y, hv.z * inv2 * wn.z, hv.w * inv2 * wn.w);
    }
    if (on)
        *reinterpret_cast<uint2*>(x_out + (size_t)r * width + i) = make_uint2(pack_bf16x2_bits(o.x, o.y), pack_bf16x2_bits(o.z, o.w));
}

// Token embedding rows (bf16) times `scale` (SCALE shader with sqrt(hidden)), f32
// residual stream h and its bf16 copy x (the input of the top PLE projection).
__global__ void __launch_bounds__(kRowThreads) embed_kernel(const uint16_t* __restrict__ table, int vocab, int width,
                                                            const int32_t* __restrict__ ids, float scale,
                                                            float* __restrict__ h, uint16_t* __restrict__ x,
                                                            uint32_t* err, int vec) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    const int id = ids[r];
    const bool ok = (unsigned)id < (unsigned)vocab;
    if (!ok && threadIdx.x == 0) raise_error(err, G4_DEVERR_BAD_INDEX);
    const uint16_t* er = table + (size_t)(ok ? id : 0) * width;
    if (vec) {  // width % 8 == 0, 16-byte aligned rows: every load of the row in flight at once
        for (int i0 = threadIdx.x * 8; i0 < width; i0 += blockDim.x * 8) {
            const uint4 e = ok ? __ldg(reinterpret_cast<const uint4*>(er + i0)) : make_uint4(0u, 0u, 0u, 0u);
            const uint32_t w[4] = {e.x, e.y, e.z, e.w};
            float v[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                v[2 * k] = bf16_bits_to_f32(w[k] & 0xFFFFu) * scale;
                v[2 * k + 1] = bf16_bits_to_f32(w[k] >> 16) * scale;
            }
            float4* hr = reinterpret_cast<float4*>(h + (size_t)r * width + i0);
            hr[0] = make_float4(v[0], v[1], v[2], v[3]);
            hr[1] = make_float4(v[4], v[5], v[6], v[7]);
            if (x)
                *reinterpret_cast<uint4*>(x + (size_t)r * width + i0) =
                    make_uint4(pack_bf16x2_bits(v[0], v[1]), pack_bf16x2_bits(v[2], v[3]), pack_bf16x2_bits(v[4], v[5]),
                               pack_bf16x2_bits(v[6], v[7]));
        }
        return;
    }
    for (int i = threadIdx.x; i < width; i += blockDim.x) {
        const float v = ok ? bf16_bits_to_f32(er[i]) * scale : 0.f;
        h[(size_t)r * width + i] = v;
        if (x) x[(size_t)r * width + i] = (uint16_t)f32_to_bf16_bits(v);
    }
}

// NORM_ROPE_SHADER for the q heads and the k head of one row, RMS_SHADER (no scale)
// for v; q goes to q_out (bf16 [rows, H, hd]); k and v are written straight into the
// bf16 caches at the row's absolute position (KVCache.append, gemma4-webgpu.js:128-135).
// Slot < H: q head, H: k, H + 1: v.

// Destination row of (row r, slot) and the output pair (i, i + hd/2) of one rotation
// pair a0 = y[i], a1 = y[i + hd/2] once the head's 1/rms is known.
// Where the K/V rows go: sequence seq's rows start at seq * cache_cap; a linear cache keeps
// position pos in row pos (pos < pos_limit), a ring cache in slot pos % ring and, for slots
// below `mirror`, again in row ring + slot.
struct KvSink {
    uint16_t *kcache, *vcache;
    int cache_cap, ring, mirror, pos_limit;
    uint32_t* err;
};
__device__ __forceinline__ uint16_t* qkv_dst(int slot, int H, int hd, int r, const G4Rows& R, int pos,
                                             uint16_t* q_out, const KvSink& kv, uint16_t** mirror_dst) {
    *mirror_dst = nullptr;
    if (slot < H) return q_out + ((size_t)r * H + slot) * hd;
    uint16_t* base = (slot == H ? kv.kcache : kv.vcache) + (size_t)row_seq(R, r) * kv.cache_cap * hd;
    if (!kv.ring) return base + (size_t)pos * hd;
    const int s = pos % kv.ring;
    if (s < kv.mirror) *mirror_dst = base + (size_t)(kv.ring + s) * hd;
    return base + (size_t)s * hd;
}
// A K/V row at or past the cache capacity is not written; it raises the device error word.
__device__ __forceinline__ bool kv_row_ok(int slot, int H, int pos, const KvSink& kv) {
    if (slot < H || (pos >= 0 && pos < kv.pos_limit)) return true;
    if (kv.err) atomicOr(kv.err, G4_DEVERR_BAD_INDEX);
    return false;
}
__device__ __forceinline__ float2 qkv_pair_s(int slot, int H, int hd, int i, float a0, float a1, float inv,
                                             float s0, float s1, int rope_angles, float rope_base, int pos) {
    if (slot == H + 1) return make_float2(a0 * inv, a1 * inv);  // v: RMS without scale (official-w4a16-layer0.js:176-182)
    const float x0 = a0 * inv * s0, x1 = a1 * inv * s1;
    float sn = 0.f, cs = 1.f;
    if (i < rope_angles) {
        const float theta = (float)pos / powf(rope_base, 2.f * (float)i / (float)hd);
        sincosf(theta, &sn, &cs);  // one argument reduction for both
    }
    return make_float2(x0 * cs - x1 * sn, x1 * cs + x0 * sn);
}
__device__ __forceinline__ float2 qkv_pair(int slot, int H, int hd, int i, float a0, float a1, float inv,
                                           const float* __restrict__ qnorm, const float* __restrict__ knorm,
                                           int rope_angles, float rope_base, int pos) {
    const float* sc = slot < H ? qnorm : knorm;
    const bool scaled = slot <= H;
    return qkv_pair_s(slot, H, hd, i, a0, a1, inv, scaled ? sc[i] : 1.f, scaled ? sc[i + (hd >> 1)] : 1.f,
                      rope_angles, rope_base, pos);
}

// Any hd % 64 == 0: one CTA per (row, head slot), thread i owns the rotation pair
// (i, i + hd/2).
__global__ void qkv_post_kernel(Planes y, int H, int hd, int has_kv,
                                const float* __restrict__ qnorm, const float* __restrict__ knorm, float eps,
                                int rope_angles, float rope_base, G4Rows R, uint16_t* __restrict__ q_out, KvSink kv) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    const int slot = blockIdx.x, r = blockIdx.y;
    const int half = hd >> 1;
    const int i = threadIdx.x;  // 0 .. half-1
    const size_t src = (size_t)r * y.ld + (size_t)slot * hd;
    const float a0 = ld_planes(y, src + i), a1 = ld_planes(y, src + i + half);
    const float inv = rsqrtf(block_sum(a0 * a0 + a1 * a1, red) / (float)hd + eps);
    const int pos = row_position(R, r);
    const float2 o = qkv_pair(slot, H, hd, i, a0, a1, inv, qnorm, knorm, rope_angles, rope_base, pos);
    if (!kv_row_ok(slot, H, pos, kv)) return;
    uint16_t* dst2;
    uint16_t* dst = qkv_dst(slot, H, hd, r, R, pos, q_out, kv, &dst2);
    const uint16_t b0 = (uint16_t)f32_to_bf16_bits(o.x), b1 = (uint16_t)f32_to_bf16_bits(o.y);
    dst[i] = b0;
    dst[i + half] = b1;
    if (dst2) {
        dst2[i] = b0;
        dst2[i + half] = b1;
    }
}

// hd = 256 * NF: one warp per (row, head slot), 8 per CTA, so a decode batch is a few
// hundred CTAs that are all resident at once (the attention behind it launches early).
// Lane l owns the float4 groups 4 (l + 32 f) .. + 3 of both halves of the head row, i.e.
// 4 NF rotation pairs.  The planes are summed in slice order with the loads of a batch
// of slices for all the lane's groups in flight together.
constexpr int kQkvWarps = 8;
template <int NF>
__global__ void __launch_bounds__(kQkvWarps * 32)
qkv_post_warp_kernel(Planes y, int H, int has_kv, int rows, const float* __restrict__ qnorm,
                     const float* __restrict__ knorm, float eps, int rope_angles, float rope_base, G4Rows R,
                     uint16_t* __restrict__ q_out, KvSink kv) {
    constexpr int hd = 256 * NF, half = hd / 2, G = 2 * NF;  // float4 groups per lane
    constexpr int PB = NF <= 2 ? 4 : 2;                        // slices per load batch
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int slots = H + (has_kv ? 2 : 0);
    const int unit = blockIdx.x * kQkvWarps + (threadIdx.x >> 5);
    const bool valid = unit < rows * slots;
    const int r = valid ? unit / slots : 0, slot = valid ? unit - r * slots : 0;
    auto goff = [&](int g) { return (g < NF ? 0 : half) + 4 * (lane + 32 * (g % NF)); };
    // The lane's norm scales (immutable) are fetched while the predecessor drains; the
    // row's position with the planes.  A warp issues in order: nothing below consumes a
    // load before every load of the row has been issued.
    float4 sc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) sc[g] = make_float4(1.f, 1.f, 1.f, 1.f);
    if (valid && slot <= H) {
        const float* nrm = slot < H ? qnorm : knorm;
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] = __ldg(reinterpret_cast<const float4*>(nrm + goff(g)));
    }
    pdl_wait();
    if (!valid) return;
    const int seq = row_seq(R, r);
    const int seq_pos = R.seq_pos ? R.seq_pos[seq] : 0;
    const float* src = y.base + (size_t)r * y.ld + (size_t)slot * hd;
    float4 a[G];
#pragma unroll
    for (int g = 0; g < G; ++g) a[g] = __ldg(reinterpret_cast<const float4*>(src + goff(g)));
    for (int s0 = 1; s0 < y.count; s0 += PB) {
        float4 b[PB][G];
#pragma unroll
        for (int k = 0; k < PB; ++k)
#pragma unroll
            for (int g = 0; g < G; ++g)
                b[k][g] = s0 + k < y.count
                              ? __ldg(reinterpret_cast<const float4*>(src + (size_t)(s0 + k) * y.stride + goff(g)))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < PB; ++k) {
            if (s0 + k < y.count) {
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    a[g].x += b[k][g].x;
                    a[g].y += b[k][g].y;
                    a[g].z += b[k][g].z;
                    a[g].w += b[k][g].w;
                }
            }
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int g = 0; g < G; ++g) ss += a[g].x * a[g].x + a[g].y * a[g].y + a[g].z * a[g].z + a[g].w * a[g].w;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = rsqrtf(ss / (float)hd + eps);
    const int pos = seq_pos + R.pos0 + r % R.rows_per_seq;
    if (!kv_row_ok(slot, H, pos, kv)) return;
    uint16_t* dst2;
    uint16_t* dst = qkv_dst(slot, H, hd, r, R, pos, q_out, kv, &dst2);
#pragma unroll
    for (int f = 0; f < NF; ++f) {
        const int i0 = 4 * (lane + 32 * f);
        const float lo[4] = {a[f].x, a[f].y, a[f].z, a[f].w}, hi[4] = {a[NF + f].x, a[NF + f].y, a[NF + f].z, a[NF + f].w};
        const float slo[4] = {sc[f].x, sc[f].y, sc[f].z, sc[f].w};
        const float shi[4] = {sc[NF + f].x, sc[NF + f].y, sc[NF + f].z, sc[NF + f].w};
        float o0[4], o1[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float2 o = qkv_pair_s(slot, H, hd, i0 + c, lo[c], hi[c], inv, slo[c], shi[c], rope_angles, rope_base,
                                        pos);
            o0[c] = o.x;
            o1[c] = o.y;
        }
        const uint2 lo2 = make_uint2(pack_bf16x2_bits(o0[0], o0[1]), pack_bf16x2_bits(o0[2], o0[3]));
        const uint2 hi2 = make_uint2(pack_bf16x2_bits(o1[0], o1[1]), pack_bf16x2_bits(o1[2], o1[3]));
        *reinterpret_cast<uint2*>(dst + i0) = lo2;
        *reinterpret_cast<uint2*>(dst + i0 + half) = hi2;
        if (dst2) {
            *reinterpret_cast<uint2*>(dst2 + i0) = lo2;
            *reinterpret_cast<uint2*>(dst2 + i0 + half) = hi2;
        }
    }
}

// GELU_MUL over a fused [gate | up] projection: out = bf16(gelu(gate) * up), four
// columns per thread (inter % 4 == 0).
__global__ void gelu_mul_kernel(Planes gu, int inter, long long n4, uint16_t* __restrict__ out) {
    pdl_trigger();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const int q = inter >> 2;
    const long long r = i / q, c = (i - r * q) * 4;
    const size_t row = (size_t)r * gu.ld;
    float4 g, u;
    ld4_planes2(gu, row + c, row + inter + c, g, u);
    *reinterpret_cast<uint2*>(out + r * inter + c) =
        make_uint2(pack_bf16x2_bits(gelu_ref(g.x) * u.x, gelu_ref(g.y) * u.y),
                   pack_bf16x2_bits(gelu_ref(g.z) * u.z, gelu_ref(g.w) * u.w));
}

// GELU_PLE: out = bf16(gelu(gate) * per_layer[row, layer, :]).
__global__ void gelu_ple_kernel(Planes gate, const float* __restrict__ per_layer, int layer, int layers, int dim,
                                long long n, uint16_t* __restrict__ out) {
    pdl_trigger();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const long long r = i / dim, d = i - r * dim;
    const float pl = per_layer[(r * layers + layer) * dim + d];  // in flight with the planes' loads
    out[i] = (uint16_t)f32_to_bf16_bits(gelu_ref(ld_planes(gate, (size_t)r * gate.ld + d)) * pl);
}

// GELU_PLE with four columns per thread (dim % 4 == 0, 16-byte aligned planes and per_layer).
__global__ void gelu_ple4_kernel(Planes gate, const float* __restrict__ per_layer, int layer, int layers, int dim,
                                 long long n4, uint16_t* __restrict__ out) {
    pdl_trigger();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const int q = dim >> 2;
    const long long r = i / q, c = (i - r * q) * 4;
    const float4 pl = *reinterpret_cast<const float4*>(per_layer + (r * layers + layer) * dim + c);  // with the planes
    const float4 g = ld4_planes(gate, (size_t)r * gate.ld + c);
    *reinterpret_cast<uint2*>(out + r * dim + c) =
        make_uint2(pack_bf16x2_bits(gelu_ref(g.x) * pl.x, gelu_ref(g.y) * pl.y),
                   pack_bf16x2_bits(gelu_ref(g.z) * pl.z, gelu_ref(g.w) * pl.w));
}

// SCALE + PLE_MIX: p = proj * proj_scale; y = (rms(p) * norm + tok_ple * sqrt(dim)) / sqrt(2)
// per (row, layer) segment of `dim`.  One CTA per segment, one thread per element.
__global__ void ple_mix_kernel(const float* __restrict__ proj, float proj_scale, const float* __restrict__ norm,
                               const float* __restrict__ tok_ple, int dim, float eps, float* __restrict__ out) {
    pdl_trigger();
    __shared__ float red[32];
    const size_t base = (size_t)blockIdx.x * dim;
    const int d = threadIdx.x;
    const float nd = __ldg(norm + d);  // immutable: fetched while the predecessor drains
    pdl_wait();
    const float tp = tok_ple[base + d];
    const float p = proj[base + d] * proj_scale;
    const float inv = rsqrtf(block_sum(p * p, red) / (float)dim + eps);
    out[base + d] = (p * inv * nd + tp * sqrtf((float)dim)) * 0.7071067811865476f;
}

// softcap + argmax, pass 1: per (row, chunk) the largest tanh(v / cap) * cap and its
// lowest index (topK keeps the first of equal values, gpu-runtime.js:1396-1425).
constexpr int kArgChunk = 4096;
__device__ __forceinline__ void arg_better(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}
__global__ void __launch_bounds__(256) argmax_partial_kernel(const float* __restrict__ logits, int vocab, float cap,
                                                             float2* __restrict__ part) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sv[256];
    __shared__ int si[256];
    const int r = blockIdx.y, c = blockIdx.x;
    const float* lr = logits + (size_t)r * vocab;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    const int end = min(vocab, (c + 1) * kArgChunk);
    for (int i = c * kArgChunk + threadIdx.x; i < end; i += blockDim.x) {
        const float raw = lr[i];
        const float v = cap > 0.f ? tanhf(raw / cap) * cap : raw;
        if (v == v) arg_better(bv, bi, v, i);  // skip NaN (topK skips non-finite logits)
    }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
        if (threadIdx.x < o) arg_better(sv[threadIdx.x], si[threadIdx.x], sv[threadIdx.x + o], si[threadIdx.x + o]);
        __syncthreads();
    }
    if (threadIdx.x == 0) part[(size_t)r * gridDim.x + c] = make_float2(sv[0], __int_as_float(si[0]));
}
// pass 2: reduce the chunk partials of a row; write the id (and optionally the value).
__global__ void __launch_bounds__(256) argmax_final_kernel(const float2* __restrict__ part, int nparts,
                                                           int32_t* __restrict__ ids, float* __restrict__ vals) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sv[256];
    __shared__ int si[256];
    const int r = blockIdx.x;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
        const float2 p = part[(size_t)r * nparts + i];
        arg_better(bv, bi, p.x, __float_as_int(p.y));
    }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
        if (threadIdx.x < o) arg_better(sv[threadIdx.x], si[threadIdx.x], sv[threadIdx.x + o], si[threadIdx.x + o]);
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        ids[r] = si[0];
        if (vals) vals[r] = sv[0];
    }
}

// Advances the positions of sequences [seq_base, seq_base + nseq) by `by`.
__global__ void advance_pos_kernel(int32_t* seq_pos, int seq_base, int nseq, int by) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < nseq) seq_pos[seq_base + i] += by;
}

inline unsigned blocks_for(long long n, int t) { return (unsigned)((n + t - 1) / t); }

// ---- the reference operators in their own form: separate f32 buffers in and out, for a
// host that keeps the reference's model graph and only swaps its runtime.

// SCALE: y = a * s.
__global__ void scale_kernel(const float* __restrict__ a, long long n, float s, float* __restrict__ y) {
    pdl_trigger();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = a[i] * s;
}

// GELU_MUL with separate gate and up buffers: y = gelu(gate) * up.
__global__ void gelu_mul_f32_kernel(const float* __restrict__ gate, const float* __restrict__ up, long long n,
                                    float* __restrict__ y) {
    pdl_trigger();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = gelu_ref(gate[i]) * up[i];
}

// GELU_PLE: y[row, d] = gelu(gate[row, d]) * ple[row, layer, d] (f32 out).
__global__ void gelu_ple_f32_kernel(const float* __restrict__ gate, const float* __restrict__ per_layer, int layer,
                                    int layers, int dim, long long n, float* __restrict__ y) {
    pdl_trigger();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const long long r = i / dim, d = i - r * dim;
    y[i] = gelu_ref(gate[i]) * per_layer[(r * layers + layer) * dim + d];
}

// NORM_ROPE: per (row, head) y = rope(x * rsqrt(mean(x^2) + eps) * scale) at position
// pos0 + row.  One CTA per (head, row), thread i owns the rotation pair (i, i + hd/2).
__global__ void norm_rope_kernel(const float* __restrict__ x, const float* __restrict__ scale, int heads, int hd,
                                 int pos0, int rope_angles, float base, float eps, float* __restrict__ y) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red[32];
    const int h = blockIdx.x, r = blockIdx.y, half = hd >> 1, i = threadIdx.x;
    const size_t src = ((size_t)r * heads + h) * hd;
    const float a0 = x[src + i], a1 = x[src + i + half];
    const float inv = rsqrtf(block_sum(a0 * a0 + a1 * a1, red) / (float)hd + eps);
    const float x0 = a0 * inv * scale[i], x1 = a1 * inv * scale[i + half];
    float sn = 0.f, cs = 1.f;
    if (i < rope_angles) {
        const float theta = (float)(pos0 + r) / powf(base, 2.f * (float)i / (float)hd);
        sn = sinf(theta);
        cs = cosf(theta);
    }
    y[src + i] = x0 * cs - x1 * sn;
    y[src + i + half] = x1 * cs + x0 * sn;
}

// The softcap of BF16_HEAD applied to logits in place: v = tanh(v / cap) * cap.
__global__ void softcap_kernel(float* __restrict__ v, long long n, float cap) {
    pdl_trigger();
    pdl_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) v[i] = tanhf(v[i] / cap) * cap;
}

}  // namespace

namespace g4 {
g4_status launch_argmax_final(g4_ctx* ctx, const float2* part, int nparts, int rows, int32_t* ids, float* vals) {
    return launch(ctx, "argmax_final_kernel", argmax_final_kernel, dim3(rows), dim3(256), 0, 1, part, nparts, ids, vals);
}
}  // namespace g4

extern "C" {

g4_status g4_rms(g4_ctx* ctx, const float* x, const float* scale, int rows, int width, float eps, void* out,
                 g4_dtype out_dtype) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (rows < 0 || width <= 0 || !x || !out) return g4::set_error(G4_ERR_INVALID, "g4_rms: bad arguments");
    if (rows == 0) return G4_OK;
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(scale) |
                         reinterpret_cast<uintptr_t>(out);
    if (width % 4 == 0 && width <= 4096 && al % 16 == 0)
        return g4::launch(ctx, "rms4_kernel", rms4_kernel, dim3(rows), dim3(((width / 4 + 31) / 32) * 32), 0, 1, x,
                          scale, width, eps, out, (int)(out_dtype == G4_BF16));
    return g4::launch(ctx, "rms_kernel", rms_kernel, dim3(rows), dim3(kRowThreads), 0, 1, x, scale, width, eps, out,
                      (int)(out_dtype == G4_BF16));
}

g4_status g4_add_scale(g4_ctx* ctx, const float* a, const float* b, long long n, float scale, float* y) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (n < 0 || !a || !b || !y) return g4::set_error(G4_ERR_INVALID, "g4_add_scale: bad arguments");
    if (n == 0) return G4_OK;
    return g4::launch(ctx, "add_scale_kernel", add_scale_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, 1, a, b, n, scale, y);
}

static Planes planes_of(const g4_planes* y) { return Planes{y->base, y->stride, y->count, y->ld}; }
static bool planes_ok(const g4_planes* y) { return y && y->base && y->count >= 1 && y->ld > 0; }

g4_status g4_post_norm_add_planes(g4_ctx* ctx, float* h, const g4_planes* y, const float* w_post, float skip,
                                  const float* w_next, int rows, int width, float eps, void* x_out_bf16) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (rows < 0 || width <= 0 || !h || !planes_ok(y) || !w_post)
        return g4::set_error(G4_ERR_INVALID, "g4_post_norm_add: bad arguments");
    if (width % 4 != 0 || width > 4096 || y->ld % 4 != 0 || (y->count > 1 && y->stride % 4 != 0))
        return g4::set_error(G4_ERR_UNSUPPORTED, "g4_post_norm_add: width %d / ldy %d (multiples of 4, width <= 4096)",
                             width, y->ld);
    if (rows == 0) return G4_OK;
    const int threads = ((width / 4 + 31) / 32) * 32;
    return g4::launch(ctx, "post_norm_add_kernel", post_norm_add_kernel, dim3(rows), dim3(threads), 0, 1, h,
                      planes_of(y), w_post, skip, w_next, width, eps, static_cast<uint16_t*>(x_out_bf16));
}

g4_status g4_post_norm_add(g4_ctx* ctx, float* h, const float* y, int ldy, const float* w_post, float skip,
                           const float* w_next, int rows, int width, float eps, void* x_out_bf16) {
    const g4_planes one{y, 1, 0, ldy};
    return g4_post_norm_add_planes(ctx, h, &one, w_post, skip, w_next, rows, width, eps, x_out_bf16);
}

g4_status g4_embed(g4_ctx* ctx, const void* table_bf16, int vocab, int width, const int32_t* ids_dev, int rows,
                   float scale, float* h_out, void* x_out_bf16) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (rows < 0 || !table_bf16 || !ids_dev || !h_out) return g4::set_error(G4_ERR_INVALID, "g4_embed: bad arguments");
    if (rows == 0) return G4_OK;
    const int vec = width % 8 == 0 && ((reinterpret_cast<uintptr_t>(table_bf16) | reinterpret_cast<uintptr_t>(h_out) |
                                         reinterpret_cast<uintptr_t>(x_out_bf16)) % 16 == 0);
    return g4::launch(ctx, "embed_kernel", embed_kernel, dim3(rows), dim3(kRowThreads), 0, 1,
                      static_cast<const uint16_t*>(table_bf16), vocab, width, ids_dev, scale, h_out,
                      static_cast<uint16_t*>(x_out_bf16), ctx->d_err, vec);
}

}  // extern "C"

namespace {

g4_status qkv_post_impl(g4_ctx* ctx, const g4_planes* y, int heads, int hd, int has_kv, const float* qnorm,
                        const float* knorm, float eps, int rope_angles, float rope_base, const G4Rows* rows_map,
                        int rows, void* q_out_bf16, void* kcache_bf16, void* vcache_bf16, int cache_cap, int ring,
                        int mirror, int pos_limit) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (rows < 0 || !planes_ok(y) || !qnorm || !rows_map || !q_out_bf16 ||
        (has_kv && (!knorm || !kcache_bf16 || !vcache_bf16)))
        return g4::set_error(G4_ERR_INVALID, "g4_qkv_post: bad arguments");
    if (hd % 64 != 0 || hd > 1024) return g4::set_error(G4_ERR_UNSUPPORTED, "g4_qkv_post: hd %d", hd);
    if (rows == 0) return G4_OK;
    const Planes P = planes_of(y);
    // the warp kernel reads float4 groups and writes 4 bf16 at a time
    const bool f4 = y->ld % 4 == 0 && (y->count == 1 || y->stride % 4 == 0) &&
                    (reinterpret_cast<uintptr_t>(y->base) & 15) == 0 && (reinterpret_cast<uintptr_t>(q_out_bf16) & 7) == 0 &&
                    (!has_kv || ((reinterpret_cast<uintptr_t>(kcache_bf16) | reinterpret_cast<uintptr_t>(vcache_bf16)) & 7) == 0);
    const long long units = (long long)rows * (heads + (has_kv ? 2 : 0));
    const dim3 wgrid((unsigned)((units + kQkvWarps - 1) / kQkvWarps)), wblock(kQkvWarps * 32);
    uint16_t* qo = static_cast<uint16_t*>(q_out_bf16);
    const KvSink kv{static_cast<uint16_t*>(kcache_bf16), static_cast<uint16_t*>(vcache_bf16), cache_cap, ring, mirror,
                    pos_limit, ctx->d_err};
    if (f4 && hd == 256)
        return g4::launch(ctx, "qkv_post_warp_kernel", qkv_post_warp_kernel<1>, wgrid, wblock, 0, 1, P, heads, has_kv,
                          rows, qnorm, knorm, eps, rope_angles, rope_base, *rows_map, qo, kv);
    if (f4 && hd == 512)
        return g4::launch(ctx, "qkv_post_warp_kernel", qkv_post_warp_kernel<2>, wgrid, wblock, 0, 1, P, heads, has_kv,
                          rows, qnorm, knorm, eps, rope_angles, rope_base, *rows_map, qo, kv);
    return g4::launch(ctx, "qkv_post_kernel", qkv_post_kernel, dim3(heads + (has_kv ? 2 : 0), rows), dim3(hd / 2), 0,
                      1, P, heads, hd, has_kv, qnorm, knorm, eps, rope_angles, rope_base, *rows_map, qo, kv);
}

}  // namespace

extern "C" {

g4_status g4_qkv_post_planes(g4_ctx* ctx, const g4_planes* y, int heads, int hd, int has_kv, const float* qnorm,
                             const float* knorm, float eps, int rope_angles, float rope_base, const G4Rows* rows_map,
                             int rows, void* q_out_bf16, void* kcache_bf16, void* vcache_bf16, int cache_cap) {
    if (has_kv && cache_cap < 1) return g4::set_error(G4_ERR_INVALID, "g4_qkv_post: cache_cap %d", cache_cap);
    return qkv_post_impl(ctx, y, heads, hd, has_kv, qnorm, knorm, eps, rope_angles, rope_base, rows_map, rows,
                         q_out_bf16, kcache_bf16, vcache_bf16, cache_cap, 0, 0, cache_cap);
}

g4_status g4_qkv_post_kv(g4_ctx* ctx, const g4_planes* y, int heads, int hd, const float* qnorm, const float* knorm,
                         float eps, int rope_angles, float rope_base, const G4Rows* rows_map, int rows,
                         void* q_out_bf16, const g4_kv* kv) {
    if (!kv)
        return qkv_post_impl(ctx, y, heads, hd, 0, qnorm, knorm, eps, rope_angles, rope_base, rows_map, rows,
                             q_out_bf16, nullptr, nullptr, 1, 0, 0, 1);
    if (hd != kv->hd) return g4::set_error(G4_ERR_INVALID, "g4_qkv_post_kv: hd %d != cache hd %d", hd, kv->hd);
    if (!rows_map || rows_map->rows_per_seq < 1) return g4::set_error(G4_ERR_INVALID, "g4_qkv_post_kv: bad row map");
    const int seq_rows = kv->ring ? kv->seq_rows : kv->rows_total;
    if (rows > 0 && (long long)(rows_map->seq_base + (rows - 1) / rows_map->rows_per_seq + 1) * seq_rows >
                        kv->rows_total)
        return g4::set_error(G4_ERR_RANGE, "g4_qkv_post_kv: sequences beyond the cache (%d rows)", kv->rows_total);
    return qkv_post_impl(ctx, y, heads, hd, 1, qnorm, knorm, eps, rope_angles, rope_base, rows_map, rows, q_out_bf16,
                         kv->k, kv->v, seq_rows, kv->ring, kv->mirror, kv->ring ? kv->capacity : seq_rows);
}

g4_status g4_qkv_post(g4_ctx* ctx, const float* y, int ldy, int heads, int hd, int has_kv, const float* qnorm,
                      const float* knorm, float eps, int rope_angles, float rope_base, const G4Rows* rows_map,
                      int rows, void* q_out_bf16, void* kcache_bf16, void* vcache_bf16, int cache_cap) {
    const g4_planes one{y, 1, 0, ldy};
    return g4_qkv_post_planes(ctx, &one, heads, hd, has_kv, qnorm, knorm, eps, rope_angles, rope_base, rows_map, rows,
                              q_out_bf16, kcache_bf16, vcache_bf16, cache_cap);
}

g4_status g4_gelu_mul_planes(g4_ctx* ctx, const g4_planes* gate_up, int rows, int inter, void* out_bf16) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (rows < 0 || inter <= 0 || !planes_ok(gate_up) || !out_bf16)
        return g4::set_error(G4_ERR_INVALID, "g4_gelu_mul: bad arguments");
    if (inter % 4 != 0 || gate_up->ld % 4 != 0 || (gate_up->count > 1 && gate_up->stride % 4 != 0))
        return g4::set_error(G4_ERR_UNSUPPORTED, "g4_gelu_mul: inter %d (multiple of 4)", inter);
    const long long n4 = (long long)rows * inter / 4;
    if (n4 == 0) return G4_OK;
    return g4::launch(ctx, "gelu_mul_kernel", gelu_mul_kernel, dim3(blocks_for(n4, 256)), dim3(256), 0, 1,
                      planes_of(gate_up), inter, n4, static_cast<uint16_t*>(out_bf16));
}

g4_status g4_gelu_mul(g4_ctx* ctx, const float* gate_up, int rows, int inter, void* out_bf16) {
    const g4_planes one{gate_up, 1, 0, 2 * inter};
    return g4_gelu_mul_planes(ctx, &one, rows, inter, out_bf16);
}

g4_status g4_gelu_ple_planes(g4_ctx* ctx, const g4_planes* gate, const float* per_layer, int layer, int layers,
                             int dim, int rows, void* out_bf16) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (rows < 0 || !planes_ok(gate) || !per_layer || !out_bf16 || layer < 0 || layer >= layers)
        return g4::set_error(G4_ERR_INVALID, "g4_gelu_ple: bad arguments");
    const long long n = (long long)rows * dim;
    if (n == 0) return G4_OK;
    const bool f4 = dim % 4 == 0 && gate->ld % 4 == 0 && (gate->count == 1 || gate->stride % 4 == 0) &&
                    ((reinterpret_cast<uintptr_t>(gate->base) | reinterpret_cast<uintptr_t>(per_layer)) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(out_bf16) & 7) == 0;
    if (f4)
        return g4::launch(ctx, "gelu_ple4_kernel", gelu_ple4_kernel, dim3(blocks_for(n / 4, 128)), dim3(128), 0, 1,
                          planes_of(gate), per_layer, layer, layers, dim, n / 4, static_cast<uint16_t*>(out_bf16));
    return g4::launch(ctx, "gelu_ple_kernel", gelu_ple_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, 1,
                      planes_of(gate), per_layer, layer, layers, dim, n, static_cast<uint16_t*>(out_bf16));
}

g4_status g4_gelu_ple(g4_ctx* ctx, const float* gate, const float* per_layer, int layer, int layers, int dim,
                      int rows, void* out_bf16) {
    const g4_planes one{gate, 1, 0, dim};
    return g4_gelu_ple_planes(ctx, &one, per_layer, layer, layers, dim, rows, out_bf16);
}

g4_status g4_ple_mix(g4_ctx* ctx, const float* proj, float proj_scale, const float* norm, const float* tok_ple,
                     int rows, int layers, int dim, float eps, float* out) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (rows < 0 || !proj || !norm || !tok_ple || !out || dim > 1024 || dim % 32)
        return g4::set_error(G4_ERR_INVALID, "g4_ple_mix: bad arguments");
    if (rows == 0) return G4_OK;
    return g4::launch(ctx, "ple_mix_kernel", ple_mix_kernel, dim3(rows * layers), dim3(dim), 0, 1, proj, proj_scale,
                      norm, tok_ple, dim, eps, out);
}

g4_status g4_softcap_argmax(g4_ctx* ctx, const float* logits, int rows, int vocab, float cap, int32_t* ids_out,
                            float* vals_out) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (rows < 0 || vocab <= 0 || !logits || !ids_out) return g4::set_error(G4_ERR_INVALID, "g4_softcap_argmax: bad arguments");
    if (rows == 0) return G4_OK;
    const int nparts = (vocab + kArgChunk - 1) / kArgChunk;
    st = g4::ensure_workspace(ctx, (size_t)rows * nparts * sizeof(float2));
    if (st) return st;
    float2* part = static_cast<float2*>(ctx->ws);
    st = g4::launch(ctx, "argmax_partial_kernel", argmax_partial_kernel, dim3(nparts, rows), dim3(256), 0, 1, logits,
                    vocab, cap, part);
    if (st) return st;
    return g4::launch(ctx, "argmax_final_kernel", argmax_final_kernel, dim3(rows), dim3(256), 0, 1,
                      static_cast<const float2*>(part), nparts, ids_out, vals_out);
}

g4_status g4_scale(g4_ctx* ctx, const float* a, long long n, float s, float* y) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (n < 0 || (n > 0 && (!a || !y))) return g4::set_error(G4_ERR_INVALID, "g4_scale: bad arguments");
    if (n == 0) return G4_OK;
    return g4::launch(ctx, "scale_kernel", scale_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, 1, a, n, s, y);
}

g4_status g4_gelu_mul_f32(g4_ctx* ctx, const float* gate, const float* up, long long n, float* y) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (n < 0 || (n > 0 && (!gate || !up || !y))) return g4::set_error(G4_ERR_INVALID, "g4_gelu_mul_f32: bad arguments");
    if (n == 0) return G4_OK;
    return g4::launch(ctx, "gelu_mul_f32_kernel", gelu_mul_f32_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, 1, gate,
                      up, n, y);
}

g4_status g4_gelu_ple_f32(g4_ctx* ctx, const float* gate, const float* per_layer, int rows, int layer, int layers,
                          int dim, float* y) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (rows < 0 || dim <= 0 || layers <= 0 || layer < 0 || layer >= layers)
        return g4::set_error(G4_ERR_INVALID, "g4_gelu_ple_f32: rows %d layer %d of %d dim %d", rows, layer, layers, dim);
    if (rows == 0) return G4_OK;
    if (!gate || !per_layer || !y) return g4::set_error(G4_ERR_INVALID, "g4_gelu_ple_f32: null argument");
    const long long n = (long long)rows * dim;
    return g4::launch(ctx, "gelu_ple_f32_kernel", gelu_ple_f32_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, 1, gate,
                      per_layer, layer, layers, dim, n, y);
}

g4_status g4_norm_rope(g4_ctx* ctx, const float* x, int rows, int heads, int hd, int pos0, const float* scale,
                       int rope_angles, float base, float eps, float* y) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (rows < 0 || heads < 1 || heads > 65535 || pos0 < 0)
        return g4::set_error(G4_ERR_INVALID, "g4_norm_rope: rows %d heads %d pos0 %d", rows, heads, pos0);
    if (hd < 64 || hd > 2048 || hd % 64 != 0)
        return g4::set_error(G4_ERR_UNSUPPORTED, "g4_norm_rope: hd %d (a multiple of 64 up to 2048)", hd);
    if (rows == 0) return G4_OK;
    if (!x || !scale || !y) return g4::set_error(G4_ERR_INVALID, "g4_norm_rope: null argument");
    return g4::launch(ctx, "norm_rope_kernel", norm_rope_kernel, dim3(heads, rows), dim3(hd / 2), 0, 1, x, scale,
                      heads, hd, pos0, rope_angles, base, eps, y);
}

g4_status g4_softcap(g4_ctx* ctx, float* logits, long long n, float cap) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (n < 0 || (n > 0 && !logits) || !(cap > 0.f))
        return g4::set_error(G4_ERR_INVALID, "g4_softcap: n %lld cap %g", n, (double)cap);
    if (n == 0) return G4_OK;
    return g4::launch(ctx, "softcap_kernel", softcap_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, 1, logits, n, cap);
}

g4_status g4_advance_positions(g4_ctx* ctx, int32_t* seq_pos, int seq_base, int nseq, int by) {
    g4_status st = g4::use_device(ctx);
    if (st) return st;
    if (!seq_pos || nseq < 0) return g4::set_error(G4_ERR_INVALID, "g4_advance_positions: bad arguments");
    if (nseq == 0) return G4_OK;
    return g4::launch(ctx, "advance_pos_kernel", advance_pos_kernel, dim3(blocks_for(nseq, 256)), dim3(256), 0, 1,
                      seq_pos, seq_base, nseq, by);
}

}  // extern "C"
