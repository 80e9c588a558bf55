// g4_common.cuh -- shared host/device helpers of libg4w4.so (sm_100a only).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>
#include <utility>
#include <vector>

#include "../../include/g4w4.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "libg4w4 is written for sm_100a only"
#endif

// ------------------------------------------------------------------ host side --

struct g4_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    int num_sms = 148;
    uint32_t* d_err = nullptr;      // device error words: [0] G4_DEVERR_* bits, [1] site of a timed-out wait
    void* ws = nullptr;             // grow-only scratch for split-K / split-KV partials
    size_t ws_bytes = 0;
    std::vector<void*> ws_retired;  // outgrown workspaces: kept until destroy (captured graphs may use them)
    void* stage = nullptr;          // grow-only staging for dtype conversions at the boundary (f32 entry points)
    size_t stage_bytes = 0;
    std::vector<void*> stage_retired;
    int32_t* d_ids = nullptr;       // staging for host token ids
    size_t d_ids_cap = 0;
    bool pdl = false;               // launch with programmatic dependent launch (g4_ctx_set_pdl)
};

// Device error word bits.
#define G4_DEVERR_TIMEOUT 1u       // a bounded mbarrier / flag wait gave up
#define G4_DEVERR_BAD_INDEX 2u     // a kernel saw an out-of-range id / position

namespace g4 {

g4_status set_error(g4_status st, const char* fmt, ...);
g4_status cuda_error(cudaError_t e, const char* what);
void count_launch(uint64_t n = 1);
// Makes ctx->device current on this thread; returns G4_OK or an error.
g4_status use_device(const g4_ctx* ctx);
// Ensures ctx->ws holds at least `bytes` (grow-only).  An outgrown buffer is retired,
// not freed, so CUDA graphs captured with it stay valid until the context is destroyed.
g4_status ensure_workspace(g4_ctx* ctx, size_t bytes);
// The same grow-only rule for ctx->stage, the bf16 copies of f32 boundary arguments.
g4_status ensure_stage(g4_ctx* ctx, size_t bytes);
// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
g4_status encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, void* base,
                               uint64_t inner, uint64_t outer, uint64_t row_pitch_bytes,
                               uint32_t box_inner, uint32_t box_outer,
                               CUtensorMapSwizzle swizzle);

// Launches `kern` on the context stream with an optional thread-block cluster along x
// and, when the context enables it, programmatic dependent launch: the kernel may start
// while its predecessor drains, and waits (griddepcontrol.wait) before it touches any
// data a predecessor produces.
template <typename... KArgs, typename... Args>
g4_status launch(g4_ctx* ctx, const char* name, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                 int cluster_x, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (cluster_x > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster_x;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    if (ctx->pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
    if (e != cudaSuccess) return cuda_error(e, name);
    count_launch();
    return G4_OK;
}

}  // namespace g4

#define G4_CHECK_CUDA(expr)                                              \
    do {                                                                 \
        cudaError_t _e = (expr);                                         \
        if (_e != cudaSuccess) return ::g4::cuda_error(_e, #expr);       \
    } while (0)

#define G4_CHECK_LAUNCH(what)                                            \
    do {                                                                 \
        cudaError_t _e = cudaGetLastError();                             \
        if (_e != cudaSuccess) return ::g4::cuda_error(_e, what);        \
        ::g4::count_launch();                                            \
    } while (0)

// ---------------------------------------------------------------- device side --

namespace g4dev {

// Round-to-nearest-even f32 -> bf16 bits by the integer rule of the reference's
// roundFloat32ToBF16 (official-w4a16.js:34-48).  Bit-identical for every input,
// NaN included, which __float2bfloat16_rn would not guarantee.
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float v) {
    uint32_t b = __float_as_uint(v);
    b += 0x7fffu + ((b >> 16) & 1u);
    return b >> 16;
}
__device__ __forceinline__ uint32_t pack_bf16x2_bits(float lo, float hi) {
    return f32_to_bf16_bits(lo) | (f32_to_bf16_bits(hi) << 16);
}
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// gelu_tanh of GELU_MUL (custom-webgpu/gpu-runtime.js:1139-1157) with the reference's clamp
// of the tanh argument to [-10, 10] (:1154).
__device__ __forceinline__ float gelu_ref(float x) {
    const float c = 0.7978845608028654f;
    const float z = c * (x + 0.044715f * x * x * x);
    const float t = tanhf(fminf(fmaxf(z, -10.f), 10.f));
    return 0.5f * x * (1.f + t);
}

// Programmatic dependent launch (no-ops when the kernel was launched without it).
// Every kernel calls pdl_trigger() first, so its successor can be scheduled early, and
// pdl_wait() before it reads or writes activations; only immutable weights may be
// fetched before the wait.  Every kernel waits, which keeps the chain transitive.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Every wait on a flag or mbarrier gives up after kWaitLimitNs of wall time (normal waits
// take microseconds); the kernel then raises G4_DEVERR_TIMEOUT and winds down.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// err[0]: G4_DEVERR_* bits; err[1]: the site code of the first wait that gave up.
__device__ __forceinline__ void raise_error(uint32_t* err, uint32_t bit, uint32_t site = 0) {
    if (!err) return;
    atomicOr(err, bit);
    if (site) atomicCAS(err + 1, 0u, site);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier helpers (shared::cta) ----
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// One poll.  A thread whose phase is not complete is suspended (it does not take issue
// slots from the warps doing work) until the phase completes or kPollSuspendNs passes.
constexpr uint32_t kPollSuspendNs = 1000000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kPollSuspendNs)
        : "memory");
    return ok != 0;
}
// Waits for the phase with `parity` to complete.  Gives up after kWaitLimitNs, raises
// G4_DEVERR_TIMEOUT (recording `site`) and returns false; the caller then winds down.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t site = 0) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    for (;;) {
        for (int i = 0; i < 4; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    raise_error(err, G4_DEVERR_TIMEOUT, site);
    return false;
}

// Warp-uniform variant: every lane of the warp gets the same answer.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t site = 0) {
    const bool ok = mbar_wait(bar, parity, err, site);
    return __all_sync(0xffffffffu, ok);
}

// ---- TMA / bulk copies ----
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// TMA tile store shared -> global (elements outside the tensor are not written), tracked as
// a bulk async-group of the issuing thread.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
                 "r"(smem_u32(smem_src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until the shared-memory sources of this thread's bulk groups have been read.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Waits until this thread's bulk groups have completed (global writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---- warp MMA (legacy HMMA path; used where the op is HBM-bound) ----
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               const uint32_t (&b)[2], const float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "f"(c[0]), "f"(c[1]),
          "f"(c[2]), "f"(c[3]));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// Offset-binary int4 pair -> exact bf16x2 (nibble - 8).  (w >> 4p) & 0x000F000F gives
// the nibbles at positions p and p+4; OR-ing 0x4300 makes bf16 128 + n, subtracting
// 136 leaves n - 8 exactly.
__device__ __forceinline__ uint32_t int4pair_to_bf16x2(uint32_t w_shifted) {
    uint32_t v;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(v) : "r"(w_shifted), "r"(0x000F000Fu), "r"(0x43004300u));
    uint32_t r;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(0x43084308u));
    return r;
}

}  // namespace g4dev
