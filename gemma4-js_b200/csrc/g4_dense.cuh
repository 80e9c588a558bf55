// g4_dense.cuh -- the tied bf16 embedding / LM head on the device (g4_head.cu, g4_decoder.cu).
#pragma once
#include "g4_common.cuh"

struct g4_dense {
    g4_ctx* ctx = nullptr;
    int K = 0, N = 0;
    uint16_t* w = nullptr;  // [N, K] bf16
    CUtensorMap bmap;       // boxes of 64 columns x 256 rows, 128B swizzle (tcgen05 B operand)
};
