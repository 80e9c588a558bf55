/*
 * g4w4.h -- C ABI of libg4w4.so, the sm_100a (B200) W4A16 hot path of gemma4-js.
 *
 * This header is the drop-in boundary.  Each entry point replaces one operator of
 * the reference's WebGPU runtime (custom-webgpu/gpu-runtime.js, "GPUOps") or of the
 * TFJS reference it was validated against; the replaced interface is cited above
 * each declaration as path:line inside the gemma4-js project.
 *
 * Conventions
 *   - Every call returns g4_status (0 = OK, negative = error) and never throws.
 *     g4_last_error_string() gives the message of the last failing call on the
 *     calling host thread (the reference's `throw new Error(...)` text).
 *   - All device work is asynchronous on the context's CUDA stream, in issue order
 *     (the reference relies on WebGPU queue order the same way).
 *   - Tensor arguments are plain device pointers unless a parameter says "host".
 *     Output buffers are caller-allocated (the reference's ops allocate their
 *     outputs; a JS shim keeps that by allocating from its own pool).
 *   - bf16 = IEEE bfloat16 bits in a uint16_t; row-major everywhere.
 *   - One context per GPU per host thread.
 */
#ifndef G4W4_H
#define G4W4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t g4_status;

#define G4_OK 0
#define G4_ERR_INVALID (-1)     /* bad shape / argument / state (reference: throw)   */
#define G4_ERR_OOM (-2)         /* cudaMalloc failed                                  */
#define G4_ERR_CUDA (-3)        /* CUDA runtime/driver error                          */
#define G4_ERR_TIMEOUT (-4)     /* a bounded device-side wait gave up                 */
#define G4_ERR_UNSUPPORTED (-5) /* valid for the reference, not implemented here      */
#define G4_ERR_RANGE (-6)       /* index out of range (token id, KV capacity)         */
#define G4_ERR_DEVICE (-7)      /* device-side check failed (bad id seen by a kernel) */

typedef enum { G4_F32 = 0, G4_BF16 = 1 } g4_dtype;

typedef struct g4_ctx g4_ctx;
typedef struct g4_linear g4_linear;
typedef struct g4_ple_table g4_ple_table;
typedef struct g4_kv g4_kv;
typedef struct g4_dense g4_dense;

/* Where the rows of a batch sit in their sequences.  Row r belongs to sequence
 * seq_base + r / rows_per_seq; its absolute position is
 *   (seq_pos ? seq_pos[seq] : 0) + pos0 + r % rows_per_seq.
 * seq_pos is a device array (one entry per sequence), so a captured decode step
 * stays valid as g4_advance_positions moves the sequences forward.
 * Prefill of one sequence s: {seq_pos, s, T, 0}; batched decode: {seq_pos, 0, 1, 0};
 * the reference's host-side position (startPos): {NULL, 0, rows, startPos}.
 * flags: G4_ROWS_HISTORY_READY (used by g4_attention_rows under programmatic dependent
 * launch) promises that seq_pos and every cache row below each row's first position
 * were written before the current CUDA graph launch, or before the last host
 * synchronisation of the stream: no kernel that may still be running writes them.
 * The attention kernel then streams that history while its predecessors drain and
 * waits for them only before q and the rows of the current positions. */
#define G4_ROWS_HISTORY_READY 1
typedef struct {
    const int32_t* seq_pos;
    int seq_base;
    int rows_per_seq;
    int pos0;
    int flags;
} g4_rows;

/* ---------------------------------------------------------------- context --
 * Replaces the WebGPU device + queue the runtime is constructed with
 * (custom-webgpu/gpu-runtime.js:1296 `new GPUOps(device)`).
 * `stream` is a cudaStream_t (NULL = the legacy default stream). */
g4_status g4_ctx_create(int device, void* stream, g4_ctx** out);
g4_status g4_ctx_destroy(g4_ctx* ctx);
g4_status g4_ctx_set_stream(g4_ctx* ctx, void* stream);
/* Programmatic dependent launch for this context's kernels (default off): each kernel
 * may be scheduled while its predecessor on the stream drains and prefetches its
 * weights before waiting for the predecessor's results.  Use it for long chains of
 * this library's kernels on one stream (a captured decode step). */
g4_status g4_ctx_set_pdl(g4_ctx* ctx, int enable);
/* Waits for all work issued on the context stream (reference: queue.onSubmittedWorkDone). */
g4_status g4_stream_sync(g4_ctx* ctx);
/* Reads and clears the device-side error word that kernels set when a bounded wait
 * times out or a kernel sees an invalid index.  Synchronises the stream.
 * *flags receives the raw bit set (0 = clean); the status is G4_ERR_TIMEOUT or
 * G4_ERR_DEVICE when a bit was set. */
g4_status g4_ctx_check_device(g4_ctx* ctx, uint32_t* flags);
/* Exercises the timeout path of the device-side bounded waits (no reference counterpart):
 * one thread waits on an mbarrier that nothing completes, through the same bounded wait
 * every kernel here uses; after about 2 s it raises G4_DEVERR_TIMEOUT with `site` and
 * returns, so g4_ctx_check_device reports G4_ERR_TIMEOUT naming the site, and the context
 * stays usable.  Nothing faults or hangs. */
g4_status g4_selftest_wait_timeout(g4_ctx* ctx, uint32_t site);
/* Message of the last failing call on this host thread ("" if none). */
const char* g4_last_error_string(void);
/* Library version string. */
const char* g4_version(void);
/* Number of kernels this library has launched in this process (all contexts). */
uint64_t g4_kernel_launch_count(void);

/* ----------------------------------------------------------- W4A16 linear --
 * g4_linear_create replaces GPUW4Linear.load (custom-webgpu/gpu-runtime.js:1385-1392),
 * which uploads `{base}.weight_packed` I32 [N, K/8] and `{base}.weight_scale`
 * BF16 [N, K/group] as raw bytes.  Same inputs and meaning: nibble j of word w of
 * row n holds column 8w+j, value (nibble - 8) (official-w4a16.js:15-19, :84-96).
 * The weights are copied (from host when src_on_device == 0) and re-laid out on
 * the device for the kernels; the caller's buffers can be freed afterwards.
 * group must be 32 (the compressed-tensors group size of the checkpoint);
 * K must be a multiple of 32. */
g4_status g4_linear_create(g4_ctx* ctx, const void* packed_i32, const void* scales_bf16,
                           int K, int N, int group, int src_on_device, g4_linear** out);
g4_status g4_linear_destroy(g4_linear* lin);
/* K, N of a linear. */
g4_status g4_linear_shape(const g4_linear* lin, int* K, int* N);

/* y[M,N] = x[M,K] . dequant(W)^T.  Replaces GPUOps.w4 (custom-webgpu/gpu-runtime.js:1316-1324,
 * W4_SHADER :1068-1102) and OfficialW4A16Linear.apply
 * (browser-tfjs-webgl-distribution/runtime/official-quantized-linear.js:82-128).
 * x bf16, FP32 accumulation, y in y_dtype (G4_BF16 or G4_F32).
 * M <= 16 runs the split-K decode GEMV; larger M runs the tcgen05 GEMM.
 * M = 0 is a no-op. */
g4_status g4_linear_w4a16(g4_ctx* ctx, const g4_linear* lin, const void* x_bf16, int M,
                          void* y, g4_dtype y_dtype);
/* GPUOps.w4 with the reference's own buffer types (custom-webgpu/gpu-runtime.js:1316-1324:
 * x is an f32 buffer [rows, inDim], the result a new f32 buffer [rows, outDim]).  x is
 * rounded to bf16 (round to nearest even) into a context staging buffer by one extra
 * kernel, then g4_linear_w4a16 runs with an f32 output.  The staging buffer grows with
 * cudaMalloc on first use of a larger M (not during stream capture). */
g4_status g4_linear_w4a16_f32(g4_ctx* ctx, const g4_linear* lin, const float* x, int M, float* y);
/* Forces one implementation (0 = auto, 1 = decode GEMV, 2 = tcgen05 GEMM) for tests
 * and benchmarks.  The GEMV accepts any M (it runs M in slices of 16). */
g4_status g4_linear_w4a16_impl(g4_ctx* ctx, const g4_linear* lin, const void* x_bf16, int M,
                               void* y, g4_dtype y_dtype, int impl);

/* The FP32 output of a linear as `count` partial planes (K split over `count` slices):
 * y[r][c] = base[0*stride + r*ld + c] + base[1*stride + r*ld + c] + ... added in slice
 * order (the same bits g4_linear_w4a16 returns with G4_F32). */
typedef struct {
    const float* base;
    int count;
    long long stride;
    int ld;
} g4_planes;
/* No reference counterpart: g4_linear_w4a16 without its last pass.  The planes live in the
 * context workspace and stay valid until the next call on this context that uses the
 * workspace (a linear, a split attention, g4_softcap_argmax); the *_planes row-wise
 * operators below read them, adding the slices on the way in. */
g4_status g4_linear_w4a16_planes(g4_ctx* ctx, const g4_linear* lin, const void* x_bf16, int M, g4_planes* out);
/* GPUOps.geluMul fused into a linear (GELU_MUL, custom-webgpu/gpu-runtime.js:1139-1157):
 * out bf16 [M, N/2] = gelu(gate) * up, for a linear whose weight rows come in slabs of
 * 128 = 64 gate rows then the 64 matching up rows (N % 128 == 0).  Same bits as
 * g4_linear_w4a16 (G4_F32) + g4_gelu_mul on the un-interleaved rows. */
g4_status g4_linear_w4a16_geglu(g4_ctx* ctx, const g4_linear* lin, const void* x_bf16, int M, void* out_bf16);
/* GPUOps.w4 followed by GPUOps.geluPle (GELU_PLE, custom-webgpu/gpu-runtime.js:1159-1173) for the
 * per-layer-input gate: out bf16 [M, N] = bf16(gelu(x . W^T) * per_layer[row, layer, :]),
 * per_layer f32 [M, layers, N].  Up to 16 rows the product goes straight from the GEMV's
 * epilogue (one launch); above, the tcgen05 GEMM's planes and g4_gelu_ple_planes (the same bits). */
g4_status g4_linear_w4a16_gelu_ple(g4_ctx* ctx, const g4_linear* lin, const void* x_bf16, int M,
                                   const float* per_layer, int layer, int layers, void* out_bf16);

/* Dequantises rows [row_start, row_start+row_count) of the weight into out
 * [row_count, K]: f32 = (nibble-8) * f32(scale) exactly as dequantizeOfficialW4A16Rows
 * (browser-tfjs-webgl-distribution/runtime/official-w4a16.js:50-101); G4_BF16 = the
 * round-to-nearest-even of that value (roundFloat32ToBF16, official-w4a16.js:34-48).
 * Reads the device layout, so it also proves the re-layout is lossless. */
g4_status g4_linear_dequant(g4_ctx* ctx, const g4_linear* lin, int row_start, int row_count,
                            void* out, g4_dtype out_dtype);

/* ------------------------------------------------------------ PLE table --
 * Replaces the shard bundle readers (custom-webgpu/gpu-runtime.js:487-527 local,
 * :798-826 remote; LocalPleW4ShardReader ple-w4-shard-reader.js:65-104).
 * packed: [vocab, width/2] bytes, low nibble = even column, two's complement
 * nibble in [-8,7] (data range [-7,7]); scales: [vocab, width/group] bf16.
 * These are the shard files' "packed block" and "scale block" with the shards of
 * row_sharded_packed_then_scales concatenated in row order.  Copied to the device. */
g4_status g4_ple_table_create(g4_ctx* ctx, const void* packed_u8, const void* scales_bf16,
                              int vocab, int width, int group, int src_on_device,
                              g4_ple_table** out);
/* Adds rows [row_start, row_start+rows) of a table created with packed_u8 == NULL
 * (one shard at a time, as the reference streams shards). */
g4_status g4_ple_table_upload_rows(g4_ctx* ctx, g4_ple_table* tab, int row_start, int rows,
                                   const void* packed_u8, const void* scales_bf16,
                                   int src_on_device);
g4_status g4_ple_table_destroy(g4_ple_table* tab);

/* out[T, width] = dequant(table[ids[t]]).  Replaces reader.pleRowsToGpu(device, ids)
 * (custom-webgpu/gpu-runtime.js:905, :993, :1050 -> _dequantRowsToGpu :265-335, WGSL :218-256).
 * ids: int32 [T], on the host (ids_on_device == 0: validated on the host, throws
 * "PLE token id out of range" like gpu-runtime.js:466-470) or on the device
 * (out-of-range ids give zero rows and raise the device error flag).
 * out_dtype G4_F32: bit-identical to q*scale (ple-w4-shard-reader.js:89-95);
 * G4_BF16: bit-identical to round-to-nearest-even of that product. */
g4_status g4_ple_gather(g4_ctx* ctx, const g4_ple_table* tab, const int32_t* ids, int T,
                        int ids_on_device, void* out, g4_dtype out_dtype);

/* -------------------------------------------------------------- KV cache --
 * Replaces KVCache (custom-webgpu/gemma4-webgpu.js:122-137): per-layer K and V
 * [capacity, hd], here in bf16.  Positions are absolute: slot = position. */
g4_status g4_kv_create(g4_ctx* ctx, int hd, int capacity, g4_kv** out);
/* A sliding-window cache that keeps only the last `ring` positions of each of `nseq`
 * sequences, as the Node reference trims its sliding-layer caches to the window
 * (node-reference/src/attention.js:299-305), instead of [capacity] rows per sequence.
 * Position p sits in slot p % ring; the cache holds nseq * (ring + 16384/hd) rows (the
 * first 16384/hd slots are repeated after the ring so that a key tile never wraps).
 * Positions still run to `capacity` (g4_kv_append's limit).  Attention on it must be
 * sliding with span + window - 1 <= ring, span = keylen - first query position (the
 * rows per sequence for g4_attention_rows, whose seq_stride must be ring + 16384/hd);
 * anything else is G4_ERR_INVALID / G4_ERR_RANGE.  ring >= 16384/hd.  g4_kv_append
 * works on single-sequence ring caches; batched ones are filled by g4_qkv_post_kv. */
g4_status g4_kv_create_ring(g4_ctx* ctx, int hd, int capacity, int ring, int nseq, g4_kv** out);
/* ring = 0 for a linear cache; seq_rows = rows per sequence of a ring cache (ring + 16384/hd),
 * or all rows of a linear one; nseq = sequences of a ring cache (1 for a linear one). */
g4_status g4_kv_layout(const g4_kv* kv, int* ring, int* seq_rows, int* nseq);
g4_status g4_kv_destroy(g4_kv* kv);
/* Appends rows of K (post k-norm + RoPE) and V (post RMS) at start_pos, which must
 * equal the cache length (gemma4-webgpu.js:128-135, same errors).  src_dtype is
 * the dtype of k and v (f32 like the reference, or bf16); the cache stores bf16. */
g4_status g4_kv_append(g4_ctx* ctx, g4_kv* kv, const void* k, const void* v, int rows,
                       int start_pos, g4_dtype src_dtype);
/* Cache length, hd and capacity. */
g4_status g4_kv_info(const g4_kv* kv, int* length, int* hd, int* capacity);
/* Resets the cache length to 0 (gemma4-webgpu.js:193-196 resetCache). */
g4_status g4_kv_reset(g4_kv* kv);
/* Device pointers of the K and V storage ([capacity, hd] bf16). */
g4_status g4_kv_buffers(const g4_kv* kv, void** k, void** v);

/* GQA attention of `rows` query rows against one KV head.  Replaces GPUOps.attention
 * (custom-webgpu/gpu-runtime.js:1357-1365: QK_SHADER :1204-1221, SOFTMAX_SHADER
 * :1223-1234, ATTN_OUT_SHADER :1236-1248) and scaledDotProductAttention
 * (browser-tfjs-webgl-distribution/runtime/official-w4a16-layer0.js:30-62).
 * q: bf16 [rows, heads, hd] (post q-norm + RoPE), out: bf16 [rows, heads, hd].
 * Logit scale 1.0.  Query row r sits at position qpos0 + r and sees keys
 * j < keylen with j <= qpos0 + r and, when sliding, j + window > qpos0 + r.
 * Requires heads <= 8, hd in {64,128,256,512}, keylen <= cache length and
 * qpos0 + rows <= keylen (every row then sees at least its own key). */
g4_status g4_attention(g4_ctx* ctx, const void* q_bf16, const g4_kv* kv, int rows, int heads,
                       int hd, int keylen, int qpos0, int sliding, int window, void* out_bf16);

/* GPUOps.attention with the reference's f32 q and f32 result (custom-webgpu/gpu-runtime.js:1357-1365,
 * `emptyF32(qrows * heads * hd)`).  The KV cache stays bf16 (g4_kv_append accepts the
 * reference's f32 K/V rows and rounds them).  q is rounded to bf16 in the context staging
 * buffer, g4_attention runs, and its bf16 rows are widened to f32 exactly: two extra
 * conversion kernels.  Same argument rules and errors as g4_attention. */
g4_status g4_attention_f32(g4_ctx* ctx, const float* q, const g4_kv* kv, int rows, int heads, int hd, int keylen,
                           int qpos0, int sliding, int window, float* out);

/* Elementwise dtype conversion of n values on the context stream, for hosts that keep the
 * reference's f32 buffers: G4_F32 -> G4_BF16 rounds to nearest even, bit-identical to
 * roundFloat32ToBF16 (browser-tfjs-webgl-distribution/runtime/official-w4a16.js:34-48);
 * G4_BF16 -> G4_F32 is exact (bits << 16, gpu-runtime.js:1058-1066); equal dtypes copy. */
g4_status g4_convert(g4_ctx* ctx, const void* src, g4_dtype src_dtype, void* dst, g4_dtype dst_dtype, long long n);

/* g4_attention for callers that cannot allocate device memory.  No counterpart in the
 * reference: its WebGPU runtime allocates a buffer for every op.  g4_attention splits a
 * long key range across CTAs and keeps the partial results in a context workspace that
 * it grows with cudaMalloc; callers whose device memory is all handed to their own pool,
 * or whose serving loop cannot absorb cudaMalloc's implicit device synchronisation, use
 * this entry point instead.  Same arguments, same checks, same result.
 *   - It allocates nothing: the partials go to one fixed 8 MiB device array compiled
 *     into the library, which every GPU that loads the library keeps until exit.
 *   - A split that needs more than 8 MiB (rows x key splits x 8 heads x (hd+2) x 4 B)
 *     is rejected with G4_ERR_RANGE and a message giving both sizes.  Single-row decode
 *     fits at every key length and head dim.
 *   - The first call on a device looks up the array's device address (with that device
 *     current), so make that first call before any stream capture.
 *   - Every call, on every context and stream of a device, shares the one array and
 *     overwrites it; calls that overlap on the GPU race.  Nothing in it needs to start
 *     at zero: each call writes every partial it reads. */
g4_status g4_attention_noalloc(g4_ctx* ctx, const void* q_bf16, const g4_kv* kv, int rows, int heads,
                               int hd, int keylen, int qpos0, int sliding, int window, void* out_bf16);

/* Attention with device-side positions (see g4_rows): row r of q attends to the cache
 * rows of its sequence, seq * seq_stride .. + keylen, keylen = seq_pos[seq] + pos0 +
 * rows_per_seq.  Same kernel and mask as g4_attention; the key split is planned for a
 * full sequence (or window), so one launch stays valid for every position. */
g4_status g4_attention_rows(g4_ctx* ctx, const void* q_bf16, const g4_kv* kv, int rows, int heads, int hd,
                            const g4_rows* map, int seq_stride, int sliding, int window, void* out_bf16);

/* ------------------------------------------------------ row-wise operators --
 * The rest of GPUOps (custom-webgpu/gpu-runtime.js:1325-1378), fused where the model
 * graph (gemma4-webgpu.js:215-310) chains them.  f32 math as in the shaders; outputs
 * that feed a W4A16 linear or the attention are bf16 (round to nearest even). */

/* GPUOps.rms (RMS_SHADER :1104-1118): out = x * rsqrt(mean(x^2) + eps) * scale (scale may be NULL). */
g4_status g4_rms(g4_ctx* ctx, const float* x, const float* scale, int rows, int width, float eps, void* out,
                 g4_dtype out_dtype);
/* GPUOps.addScale (ADD_SCALE :1120-1128): y = (a + b) * scale. */
g4_status g4_add_scale(g4_ctx* ctx, const float* a, const float* b, long long n, float scale, float* y);
/* GPUOps.scale (SCALE_SHADER :1130-1137): y = a * s. */
g4_status g4_scale(g4_ctx* ctx, const float* a, long long n, float s, float* y);
/* GPUOps.geluMul (GELU_MUL :1139-1157) on the reference's separate f32 gate and up buffers:
 * y = gelu_tanh(gate) * up, tanh argument clamped to [-10, 10], f32 out. */
g4_status g4_gelu_mul_f32(g4_ctx* ctx, const float* gate, const float* up, long long n, float* y);
/* GPUOps.geluPle (GELU_PLE :1159-1173) with f32 out: y[r, d] = gelu(gate[r, d]) * ple[r, layer, d]
 * (ple f32 [rows, layers, dim]). */
g4_status g4_gelu_ple_f32(g4_ctx* ctx, const float* gate, const float* per_layer, int rows, int layer, int layers,
                          int dim, float* y);
/* GPUOps.normRope (NORM_ROPE_SHADER :1175-1202): per row r and head, RMS-normalise the
 * head's hd values (eps), multiply by scale[hd], then rotate pairs (i, i + hd/2) for
 * i < rope_angles (= floor(ropeProp * hd / 2)) by theta = (pos0 + r) / base^(2i/hd).
 * x, y f32 [rows, heads, hd]; hd a multiple of 64. */
g4_status g4_norm_rope(g4_ctx* ctx, const float* x, int rows, int heads, int hd, int pos0, const float* scale,
                       int rope_angles, float base, float eps, float* y);
/* The softcap of BF16_HEAD (:1265-1277, `tanh(raw / softcap) * softcap`) applied in place to
 * logits from g4_dense_matmul (GPUOps.headChunk = g4_dense_matmul + g4_softcap). */
g4_status g4_softcap(g4_ctx* ctx, float* logits, long long n, float cap);
/* rms + addScale (+ the next rms) of one residual update (gemma4-webgpu.js:264-273, :288-297, :302-307):
 * h = (h + rms(y) * w_post) * skip; x_out = bf16(w_next ? rms(h) * w_next : h) (x_out may be NULL). */
g4_status g4_post_norm_add(g4_ctx* ctx, float* h, const float* y, int ldy, const float* w_post, float skip,
                           const float* w_next, int rows, int width, float eps, void* x_out_bf16);
/* Embedding rows times scale (gemma4-webgpu.js:199, :318 scale by sqrt(hidden)): h f32, x bf16 (may be NULL).
 * ids on the device; an out-of-range id gives a zero row and raises the device error word. */
g4_status g4_embed(g4_ctx* ctx, const void* table_bf16, int vocab, int width, const int32_t* ids_dev, int rows,
                   float scale, float* h_out, void* x_out_bf16);
/* GPUOps.normRope (NORM_ROPE_SHADER :1175-1202) for the q heads and the k head, rms without scale
 * for v, and KVCache.append (gemma4-webgpu.js:238-249): y f32 [rows, ldy] holds q (heads*hd),
 * then k (hd), then v (hd); q_out bf16 [rows, heads, hd]; k and v go to the bf16 caches at
 * row seq * cache_cap + position.  has_kv = 0 processes q only (KV-shared layers). */
g4_status g4_qkv_post(g4_ctx* ctx, const float* y, int ldy, int heads, int hd, int has_kv, const float* qnorm,
                      const float* knorm, float eps, int rope_angles, float rope_base, const g4_rows* map,
                      int rows, void* q_out_bf16, void* kcache_bf16, void* vcache_bf16, int cache_cap);
/* GPUOps.geluMul (GELU_MUL :1139-1157) over a fused [gate | up] projection [rows, 2*inter] -> bf16 [rows, inter]. */
g4_status g4_gelu_mul(g4_ctx* ctx, const float* gate_up, int rows, int inter, void* out_bf16);
/* GPUOps.geluPle (GELU_PLE :1159-1173): bf16(gelu(gate) * per_layer[row, layer, :]). */
g4_status g4_gelu_ple(g4_ctx* ctx, const float* gate, const float* per_layer, int layer, int layers, int dim,
                      int rows, void* out_bf16);
/* The same four operators reading a linear's output as g4_planes (the row pitch is
 * planes->ld; no reference counterpart beyond their plain forms). */
g4_status g4_post_norm_add_planes(g4_ctx* ctx, float* h, const g4_planes* y, const float* w_post, float skip,
                                  const float* w_next, int rows, int width, float eps, void* x_out_bf16);
g4_status g4_qkv_post_planes(g4_ctx* ctx, const g4_planes* y, int heads, int hd, int has_kv, const float* qnorm,
                             const float* knorm, float eps, int rope_angles, float rope_base, const g4_rows* map,
                             int rows, void* q_out_bf16, void* kcache_bf16, void* vcache_bf16, int cache_cap);
/* g4_qkv_post_planes writing K and V into a cache object (linear or ring): row r's K/V go to
 * sequence seq(r)'s rows (seq * seq_rows, g4_kv_layout) at slot position (linear) or
 * position % ring (ring, with the mirrored copy).  kv = NULL processes q only (KV-shared
 * layers).  A position at or past the cache capacity raises G4_DEVERR_BAD_INDEX on the
 * device and writes no K/V. */
g4_status g4_qkv_post_kv(g4_ctx* ctx, const g4_planes* y, int heads, int hd, const float* qnorm, const float* knorm,
                         float eps, int rope_angles, float rope_base, const g4_rows* map, int rows, void* q_out_bf16,
                         const g4_kv* kv);
g4_status g4_gelu_mul_planes(g4_ctx* ctx, const g4_planes* gate_up, int rows, int inter, void* out_bf16);
g4_status g4_gelu_ple_planes(g4_ctx* ctx, const g4_planes* gate, const float* per_layer, int layer, int layers,
                             int dim, int rows, void* out_bf16);
/* GPUOps.scale + GPUOps.pleMix (SCALE :1130-1137, PLE_MIX :1250-1263, gemma4-webgpu.js:318-321):
 * out = (rms(proj * proj_scale) * norm + tok_ple * sqrt(dim)) / sqrt(2) per [row, layer] segment. */
g4_status g4_ple_mix(g4_ctx* ctx, const float* proj, float proj_scale, const float* norm, const float* tok_ple,
                     int rows, int layers, int dim, float eps, float* out);
/* Softcap and greedy pick (BF16_HEAD's tanh(x/cap)*cap :1275, topK :1396-1425 and
 * gemma4-webgpu.js:465-478): per row the lowest index of the largest capped logit
 * (non-finite logits skipped); vals_out may be NULL.  cap <= 0 disables the softcap. */
g4_status g4_softcap_argmax(g4_ctx* ctx, const float* logits, int rows, int vocab, float cap, int32_t* ids_out,
                            float* vals_out);
/* seq_pos[seq_base .. seq_base + nseq) += by (device-side step counter of a decode loop). */
g4_status g4_advance_positions(g4_ctx* ctx, int32_t* seq_pos, int seq_base, int nseq, int by);

/* ------------------------------------------------------- bf16 dense (LM head) --
 * The tied bf16 embedding used as the LM head (gemma4-webgpu.js:170-188, BF16_HEAD
 * :1265-1277): w bf16 [N, K], copied to the device (NULL w: allocate only). */
g4_status g4_dense_create(g4_ctx* ctx, const void* w_bf16, int K, int N, int src_on_device, g4_dense** out);
g4_status g4_dense_destroy(g4_dense* d);
/* Device pointer of the [N, K] bf16 weights (the embedding table for g4_embed). */
g4_status g4_dense_weights(const g4_dense* d, void** w);
/* y[M, N] f32 = x[M, K] bf16 . W^T (headChunk without the softcap, all chunks in one launch). */
g4_status g4_dense_matmul(g4_ctx* ctx, const g4_dense* d, const void* x_bf16, int M, float* y);
/* Logits, softcap and greedy pick in one pass, without materialising the [M, N] logits:
 * ids_out[m] (and vals_out[m], may be NULL) as g4_dense_matmul followed by
 * g4_softcap_argmax (same bits: the same tensor-core accumulation order).  No reference
 * counterpart beyond those two; uses the context workspace for [M, 2*ceil(N/256)] pairs. */
g4_status g4_dense_argmax(g4_ctx* ctx, const g4_dense* d, const void* x_bf16, int M, float cap, int32_t* ids_out,
                          float* vals_out);

/* ------------------------------------------------- persistent batch-1 decoder --
 * The whole greedy decode step of one sequence (Gemma4WebGPU.forward + logits + greedy,
 * custom-webgpu/gemma4-webgpu.js:311-480: every layer's encodeLayer :215-310 over the
 * operators above) as ONE kernel launch with one CTA per SM: phases separated by grid-wide
 * barriers, each CTA streaming its share of the next linear's int4 weights into shared
 * memory while the barrier before it resolves.  The arithmetic is the op path's (exact
 * int4 x bf16 products, FP32 accumulation, bf16 activations into the linears, f32 norms);
 * only summation orders differ.  Built from the same objects the op path uses. */
typedef struct g4_decoder g4_decoder;
typedef struct {
    const g4_linear *qkv, *o, *gu, *down, *pg, *pp; /* gu: gate/up rows in 64-row slabs (g4_linear_w4a16_geglu) */
    const float *n_in, *n_pa, *n_pf, *n_pff, *n_pple, *qn, *kn; /* f32 norm scales (kn unused without has_kv) */
    float skip;               /* layer scalar of the PLE residual */
    const g4_kv* kv;          /* this layer's cache, or the cache it shares */
    int has_kv;               /* 0: a KV-shared layer (reads kv, appends nothing) */
    int full;                 /* 1: global attention; 0: sliding window */
    int rope_angles;          /* floor(rope proportion * hd / 2) */
    float rope_base;
    int inter;                /* MLP width (gu has 2 * inter rows) */
} g4_decoder_layer;
typedef struct {
    int layers, hidden, heads, ple_dim, window, vocab;
    float eps, softcap;
    const g4_linear* top;      /* per_layer_model_projection [layers * ple_dim, hidden] */
    const float* ple_norm;     /* [ple_dim] */
    const float* final_norm;   /* [hidden] */
    const g4_dense* embed;     /* tied bf16 embedding [vocab, hidden], also the LM head */
    const g4_ple_table* ple;   /* [vocab, layers * ple_dim] */
} g4_decoder_desc;
/* No reference counterpart (the reference dispatches each operator).  Validates the shapes,
 * plans each CTA's share of every linear and allocates the decoder's device scratch.
 * G4_ERR_UNSUPPORTED when a CTA's share of a linear does not fit its shared memory or the
 * caches are longer than 256 key tiles (16384 positions at head dim 256). */
g4_status g4_decoder_create(g4_ctx* ctx, const g4_decoder_desc* desc, const g4_decoder_layer* layers,
                            g4_decoder** out);
g4_status g4_decoder_destroy(g4_decoder* dec);
/* One greedy decode step of sequence 0 (cache rows = positions): reads the token ids[0] and the
 * position seq_pos[0] (device), appends K/V at that position in every layer with has_kv,
 * writes the next token to next[0] (its capped logit to val[0] if val is not NULL) and
 * advances seq_pos[0].  ids and next may be the same buffer, so a CUDA graph of this call
 * replays step after step.  A cooperative launch of one CTA per SM: no other kernel of the
 * device may hold SMs it needs for the length of the step. */
g4_status g4_decoder_step(g4_ctx* ctx, g4_decoder* dec, const int32_t* ids, int32_t* seq_pos, int32_t* next,
                          float* val);
/* After a step reported G4_ERR_TIMEOUT (g4_ctx_check_device): clears the decoder's grid
 * barrier words so the next step starts clean.  Synchronises the context stream. */
g4_status g4_decoder_reset(g4_decoder* dec);
/* Tracing hook (no reference counterpart): while timeline is set, every step writes globaltimer
 * stamps (ns) into that device buffer, `entries` per CTA (row c of a [CTAs][entries] array;
 * the step runs one CTA per SM): the start, then in program order a (weights ready, linear done)
 * pair per linear, an (arrive, pass) pair per grid barrier, four stamps per layer's attention
 * tile (requested, q ready, K/V in, done; all four at once without a tile) and one after each
 * row-wise operator (combine, attention load, norms, activation load, PLE mix), then the end.  NULL switches it off.  A step already captured in a CUDA
 * graph keeps the setting it was captured with. */
g4_status g4_decoder_set_timeline(g4_decoder* dec, unsigned long long* timeline, int entries);

#ifdef __cplusplus
}
#endif
#endif /* G4W4_H */
