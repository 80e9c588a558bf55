// g4_glue.cuh -- row-to-sequence position map shared by the fused row-wise kernels and
// the attention (the public struct is g4_rows in include/g4w4.h).
#pragma once
#include "g4_common.cuh"

using G4Rows = g4_rows;
