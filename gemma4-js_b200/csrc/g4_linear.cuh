// g4_linear.cuh -- device layout of a W4A16 linear, shared by the GEMV and the GEMM.
#pragma once
#include "g4_common.cuh"

struct g4_linear_dev {
    int K = 0, N = 0;
    int Kc = 0;              // ceil(K / 64): 512-byte blocks per 16-row tile
    int NT = 0;              // ceil(N / 16): 16-row tiles
    uint4* wfrag = nullptr;  // [NT][Kc][32] uint4
    uint2* sfrag = nullptr;  // [NT][Kc][8]  uint2 (4 bf16 scales)
};

struct g4_linear {
    g4_ctx* ctx = nullptr;
    g4_linear_dev dev;
    CUtensorMap wmap;  // wfrag as uint32 [NT][Kc*128], boxes of 16 tiles x one 512-byte block
    CUtensorMap smap;  // sfrag as uint32 [NT][Kc*16],  boxes of 16 tiles x one 64-byte block
};

namespace g4 {
g4_status launch_gemv(g4_ctx* ctx, const g4_linear* lin, const uint16_t* x, int M, void* y, int y_f32);
// tcgen05 prefill GEMM (g4_gemm_sm100.cu)
bool gemm_supported(const g4_linear* lin, int M);
g4_status launch_gemm(g4_ctx* ctx, const g4_linear* lin, const uint16_t* x, int M, void* y, int y_f32);
g4_status make_linear_maps(g4_linear* lin);
// tcgen05 GEMM with a bf16 B operand loaded by TMA (bmap: [N, K] bf16, boxes of 64 x 256,
// 128B swizzle); y f32 [M, N].
g4_status launch_gemm_bf16(g4_ctx* ctx, const CUtensorMap& bmap, int N, int K, const uint16_t* x, int M, float* y);
}  // namespace g4
