// g4_attention.cuh -- KV cache object shared by the attention kernels.
#pragma once
#include "g4_common.cuh"

struct g4_kv {
    g4_ctx* ctx = nullptr;
    int hd = 0, capacity = 0, length = 0;
    int rows_total = 0;         // rows covered by the tensor maps
    uint16_t* k = nullptr;      // [capacity, hd] bf16
    uint16_t* v = nullptr;
    CUtensorMap kmap, vmap;     // 128B-swizzled boxes of 64 columns x (16384/hd) rows
    CUtensorMap kmap_narrow, vmap_narrow;  // the same with boxes of (8192/hd) rows
};

namespace g4 {
g4_status make_kv_maps(g4_kv* kv);
g4_status launch_attention(g4_ctx* ctx, const g4_kv* kv, int kv_row0, const uint16_t* q, int rows,
                           int heads, int keylen, int qpos0, int sliding, int window, uint16_t* out,
                           void* fixed_scratch = nullptr, size_t fixed_bytes = 0, const g4_rows* map = nullptr,
                           int seq_stride = 0);
}  // namespace g4
