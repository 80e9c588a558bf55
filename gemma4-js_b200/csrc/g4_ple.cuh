// g4_ple.cuh -- the device-resident PLE W4 table (shared by the gather and the decoder).
#pragma once
#include "g4_common.cuh"

struct g4_ple_table {
    g4_ctx* ctx = nullptr;
    int vocab = 0, width = 0, group = 0;
    uint8_t* packed = nullptr;   // [vocab, width/2]: low nibble = even column, two's complement
    uint16_t* scales = nullptr;  // [vocab, width/group] bf16 bits
};
