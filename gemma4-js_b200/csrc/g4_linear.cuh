// g4_linear.cuh -- device layout of a W4A16 linear, shared by the GEMV and the GEMM.
#pragma once
#include "g4_common.cuh"

struct g4_linear_dev {
    int K = 0, N = 0;
    int Kc = 0;              // ceil(K / 64): 512-byte blocks per 16-row tile
    int NT = 0;              // ceil(N / 16): 16-row tiles
    uint4* wfrag = nullptr;  // [NT][Kc][32] uint4
    uint2* sfrag = nullptr;  // [NT][Kc][8]  uint2 (4 bf16 scales)
    // GEMM layout: [NS][Kc] blocks of kTblkBytes, one per 128-row slab and 64-column step:
    // nibbles [2 halves][128 rows][16 B] (row r, columns 32h .. 32h+31 of the step, words
    // in column order, nibbles within a word permuted as in wfrag), then scales
    // [2 halves][128 rows] bf16.  Rows past N and columns past K hold q = 0, scale 0.
    int NS = 0;              // ceil(N / 128)
    uint8_t* tblk = nullptr;
};

struct g4_linear {
    g4_ctx* ctx = nullptr;
    g4_linear_dev dev;
};

namespace g4 {
constexpr int kTblkBytes = 2 * 128 * 16 + 2 * 128 * 2;  // 4608
g4_status launch_gemv(g4_ctx* ctx, const g4_linear* lin, const uint16_t* x, int M, void* y, int y_f32,
                      const float* ple = nullptr, int ple_ld = 0);
// tcgen05 W4A16 GEMM, weights dequantised into tensor memory (g4_gemm_w4.cu)
bool gemm_supported(const g4_linear* lin, int M);
g4_status launch_gemm(g4_ctx* ctx, const g4_linear* lin, const uint16_t* x, int M, void* y, int y_f32);
// The f32 output left as partial planes in the context workspace (see g4_planes).
g4_status launch_gemm_planes(g4_ctx* ctx, const g4_linear* lin, const uint16_t* x, int M, g4_planes* planes);
// GeGLU of a linear whose 128-row slabs are 64 gate rows then the 64 matching up rows:
// out bf16 [M, N/2] (fused into the GEMM epilogue when the tiles are not split).
g4_status launch_gemm_geglu(g4_ctx* ctx, const g4_linear* lin, const uint16_t* x, int M, uint16_t* out);
g4_status launch_geglu_planes(g4_ctx* ctx, const g4_planes& pl, int M, int N, uint16_t* out);
// tcgen05 GEMM with a bf16 B operand loaded by TMA (bmap: [N, K] bf16, boxes of 64 x 256,
// 128B swizzle); y f32 [M, N].
g4_status launch_gemm_bf16(g4_ctx* ctx, const CUtensorMap& bmap, int N, int K, const uint16_t* x, int M, float* y);
}  // namespace g4
