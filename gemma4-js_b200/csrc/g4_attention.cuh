// g4_attention.cuh -- KV cache object shared by the attention kernels.
#pragma once
#include "g4_common.cuh"

// Linear cache (g4_kv_create): slot = position, rows_total = capacity rows; a batch of
// sequences shares one such cache with a caller-chosen row stride per sequence.
// Ring cache (g4_kv_create_ring), for sliding-window layers: each of nseq sequences owns
// seq_rows = ring + mirror rows; position p lives in slot p % ring, and slots 0..mirror-1
// are written twice, the second copy in rows ring..ring+mirror-1, so that a key tile of up
// to `mirror` rows that starts at any slot reads contiguous rows (one TMA box, no split
// at the wrap).  mirror = 16384 / hd, the widest key tile of the attention kernels.
struct g4_kv {
    g4_ctx* ctx = nullptr;
    int hd = 0, capacity = 0, length = 0;
    int rows_total = 0;         // rows covered by the tensor maps
    int ring = 0;               // 0: linear; > 0: slots per sequence
    int mirror = 0;             // ring caches: rows repeated after the ring
    int nseq = 1;               // ring caches: sequences
    int seq_rows = 0;           // ring caches: rows per sequence (ring + mirror)
    uint16_t* k = nullptr;      // [rows_total, hd] bf16
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
