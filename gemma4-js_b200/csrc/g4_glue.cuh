// g4_glue.cuh -- row-to-sequence position map shared by the fused row-wise kernels and
// the attention (the public struct is g4_rows in include/g4w4.h).
#pragma once
#include "g4_common.cuh"

using G4Rows = g4_rows;

namespace g4 {
// Pass 2 of the greedy pick: per row, the lowest index of the largest of `nparts` partial
// (value, index-as-float-bits) pairs; ids (and vals if not NULL) out.
g4_status launch_argmax_final(g4_ctx* ctx, const float2* part, int nparts, int rows, int32_t* ids, float* vals);
}  // namespace g4
