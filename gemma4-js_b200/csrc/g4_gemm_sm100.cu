// g4_gemm_sm100.cu -- tcgen05 prefill GEMM (placeholder until the kernel lands).
#include "g4_linear.cuh"

namespace g4 {
bool gemm_supported(const g4_linear*, int) { return false; }
g4_status launch_gemm(g4_ctx*, const g4_linear*, const uint16_t*, int, void*, int) {
    return set_error(G4_ERR_UNSUPPORTED, "tcgen05 GEMM not built");
}
}  // namespace g4
