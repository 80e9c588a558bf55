/*
 * g4_oracle.h -- CPU restatement of the gemma4-js W4A16 hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker the CUDA path is compared with
 * and the timed CPU baseline; the product (libg4w4.so) never links or calls it.
 *
 * The reference path is JavaScript run by @tensorflow/tfjs (no node runtime and no
 * tfjs exist on this machine or on the GPU boxes), so each function restates the
 * cited JS in plain C with the same f32 arithmetic.  Citations are path:line inside
 * the gemma4-js project.
 */
#ifndef G4_ORACLE_H
#define G4_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* roundFloat32ToBF16 (browser-tfjs-webgl-distribution/runtime/official-w4a16.js:34-48). */
uint16_t g4o_f32_to_bf16_bits(float v);
float g4o_round_f32_to_bf16(float v);
float g4o_bf16_bits_to_f32(uint16_t b);

/* dequantizeOfficialW4A16Rows (official-w4a16.js:50-101); returns 0 or -1 on bad shapes. */
int g4o_dequant_w4a16_rows(const int32_t* packed, const uint16_t* scales_bf16, int out_dim,
                           int in_dim, int row_start, int row_count, int group, float* out);

/* OfficialW4A16Linear.apply (official-quantized-linear.js:82-128): dequantise 256 output
 * rows at a time, then y = x . W^T in f32.  x f32 [M,K], y f32 [M,N].
 * nthreads > 1 splits the output chunks over pthreads (CPU baseline only). */
/* g4o_dequant_w4a16_rows over all N rows, split over nthreads host threads. */
int g4o_dequant_w4a16_par(const int32_t* packed, const uint16_t* scales_bf16, int N, int K, int group,
                          float* out, int nthreads);
int g4o_linear_w4a16(const float* x, int M, const int32_t* packed, const uint16_t* scales_bf16,
                     int K, int N, int group, float* y, int nthreads);

/* LocalPleW4ShardReader.readRows (browser-tfjs-webgl-distribution/runtime/ple-w4-shard-reader.js:65-104)
 * over a de-sharded table: packed [vocab, width/2] bytes, scales [vocab, width/group] bf16.
 * Returns -2 (the reference throws "PLE token out of range") on a bad id. */
int g4o_ple_read_rows(const uint8_t* packed, const uint16_t* scales_bf16, int vocab, int width,
                      int group, const int32_t* ids, int T, float* out, int nthreads);
/* Same, rounded to bf16 with roundFloat32ToBF16. */
int g4o_ple_read_rows_bf16(const uint8_t* packed, const uint16_t* scales_bf16, int vocab,
                           int width, int group, const int32_t* ids, int T, uint16_t* out,
                           int nthreads);

/* GPUOps.attention (custom-webgpu/gpu-runtime.js:1204-1248, :1357-1365) with the mask of
 * scaledDotProductAttention (official-w4a16-layer0.js:30-62): q f32 [rows, heads, hd],
 * kc/vc f32 [keylen.., hd] (one KV head), out f32 [rows, heads, hd]. */
int g4o_attention(const float* q, const float* kc, const float* vc, int rows, int heads, int hd,
                  int keylen, int qpos0, int sliding, int window, float* out);

#ifdef __cplusplus
}
#endif
#endif
