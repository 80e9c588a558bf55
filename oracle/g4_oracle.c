/*
 * g4_oracle.c -- CPU restatement of the gemma4-js W4A16 hot path (see g4_oracle.h).
 *
 * TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference arm of bench.py, never by the product library.
 *
 * Parity pins: the PLE decode and the bf16 rounding are checked against vectors
 * produced by the reference's own Python quantiser (tools/build_ple_w4_full.py,
 * tests/golden/make_golden.py).  The linear dequant and attention follow the JS by
 * restatement only (no JS runtime exists here), so those two are pinned to the
 * cited source lines, not to executed reference output.
 */
#include "g4_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* official-w4a16.js:34-48: add 0x7fff + lsb, truncate the low 16 bits. */
uint16_t g4o_f32_to_bf16_bits(float v) {
    uint32_t bits;
    memcpy(&bits, &v, 4);
    uint32_t lsb = (bits >> 16) & 1u;
    bits = bits + 0x7fffu + lsb;
    return (uint16_t)(bits >> 16);
}

float g4o_bf16_bits_to_f32(uint16_t b) {
    /* ple-w4-shard-reader.js:2-7 and gpu-runtime.js:1058-1066: bits << 16. */
    uint32_t u = ((uint32_t)b) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float g4o_round_f32_to_bf16(float v) { return g4o_bf16_bits_to_f32(g4o_f32_to_bf16_bits(v)); }

/* official-w4a16.js:15-19: offset-binary nibble -> [-8, 7]. */
static inline int signed_int4_from_nibble(uint32_t nibble) { return (int)(nibble & 0x0fu) - 8; }

/* official-w4a16.js:50-101. */
int g4o_dequant_w4a16_rows(const int32_t* packed, const uint16_t* scales_bf16, int out_dim,
                           int in_dim, int row_start, int row_count, int group, float* out) {
    if (in_dim % 8 != 0 || group <= 0 || in_dim % group != 0) return -1;
    if (row_start < 0 || row_count < 0 || row_start + row_count > out_dim) return -1;
    const int packed_in = in_dim / 8;
    const int groups_per_row = in_dim / group;
    for (int local = 0; local < row_count; ++local) {
        const int row = row_start + local;
        const int32_t* prow = packed + (size_t)row * packed_in;
        const uint16_t* srow = scales_bf16 + (size_t)row * groups_per_row;
        float* orow = out + (size_t)local * in_dim;
        for (int pc = 0; pc < packed_in; ++pc) {
            const uint32_t word = (uint32_t)prow[pc];
            for (int k = 0; k < 8; ++k) {
                const int idx = pc * 8 + k;
                const int q = signed_int4_from_nibble(word >> (k * 4));
                const float scale = g4o_bf16_bits_to_f32(srow[idx / group]);
                orow[idx] = (float)q * scale; /* exact in f32 */
            }
        }
    }
    return 0;
}

typedef struct {
    const int32_t* packed;
    const uint16_t* scales;
    int N, K, group, t, nt;
    float* out;
} dequant_job;

static void* dequant_worker(void* arg) {
    dequant_job* j = (dequant_job*)arg;
    const int r0 = (int)((long long)j->N * j->t / j->nt), r1 = (int)((long long)j->N * (j->t + 1) / j->nt);
    g4o_dequant_w4a16_rows(j->packed, j->scales, j->N, j->K, r0, r1 - r0, j->group, j->out + (size_t)r0 * j->K);
    return NULL;
}

/* official-quantized-linear.js:100-111 for a whole weight: every row dequantised to f32 once,
 * rows split over nthreads host threads (the same values as g4o_dequant_w4a16_rows). */
int g4o_dequant_w4a16_par(const int32_t* packed, const uint16_t* scales_bf16, int N, int K, int group,
                          float* out, int nthreads) {
    if (K % 8 != 0 || group <= 0 || K % group != 0 || N < 0) return -1;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > N) nthreads = N > 0 ? N : 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
    dequant_job* jobs = (dequant_job*)malloc(sizeof(dequant_job) * nthreads);
    if (!th || !jobs) {
        free(th);
        free(jobs);
        return -3;
    }
    for (int i = 0; i < nthreads; ++i) {
        dequant_job j = {packed, scales_bf16, N, K, group, i, nthreads, out};
        jobs[i] = j;
        pthread_create(&th[i], NULL, dequant_worker, &jobs[i]);
    }
    for (int i = 0; i < nthreads; ++i) pthread_join(th[i], NULL);
    free(th);
    free(jobs);
    return 0;
}

typedef struct {
    const float* x;
    int M, K, N, group;
    const int32_t* packed;
    const uint16_t* scales;
    float* y;
    int chunk0, chunk_step;
} linear_job;

#define G4O_OUTPUT_CHUNK 256 /* official-quantized-linear.js:13 outputChunkSize */

static void* linear_worker(void* arg) {
    linear_job* j = (linear_job*)arg;
    const int K = j->K;
    float* w = (float*)malloc((size_t)G4O_OUTPUT_CHUNK * K * sizeof(float));
    if (!w) return (void*)1;
    for (int c = j->chunk0; c * G4O_OUTPUT_CHUNK < j->N; c += j->chunk_step) {
        const int row_start = c * G4O_OUTPUT_CHUNK;
        const int rows = (j->N - row_start) < G4O_OUTPUT_CHUNK ? (j->N - row_start) : G4O_OUTPUT_CHUNK;
        /* official-quantized-linear.js:103-111: dequantise the chunk to f32 */
        g4o_dequant_w4a16_rows(j->packed, j->scales, j->N, K, row_start, rows, j->group, w);
        /* :113-117: tf.matMul(x, w, false, true) in f32 */
        for (int m = 0; m < j->M; ++m) {
            const float* xr = j->x + (size_t)m * K;
            for (int r = 0; r < rows; ++r) {
                const float* wr = w + (size_t)r * K;
                float acc = 0.f;
                for (int k = 0; k < K; ++k) acc += xr[k] * wr[k];
                j->y[(size_t)m * j->N + row_start + r] = acc;
            }
        }
    }
    free(w);
    return NULL;
}

int g4o_linear_w4a16(const float* x, int M, const int32_t* packed, const uint16_t* scales_bf16,
                     int K, int N, int group, float* y, int nthreads) {
    if (K % 8 != 0 || group <= 0 || K % group != 0 || M < 0 || N < 0) return -1;
    if (nthreads < 1) nthreads = 1;
    linear_job base = {x, M, K, N, group, packed, scales_bf16, y, 0, nthreads};
    if (nthreads == 1) return linear_worker(&base) ? -3 : 0;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
    linear_job* jobs = (linear_job*)malloc(sizeof(linear_job) * nthreads);
    int rc = 0;
    for (int i = 0; i < nthreads; ++i) {
        jobs[i] = base;
        jobs[i].chunk0 = i;
        pthread_create(&th[i], NULL, linear_worker, &jobs[i]);
    }
    for (int i = 0; i < nthreads; ++i) {
        void* r = NULL;
        pthread_join(th[i], &r);
        if (r) rc = -3;
    }
    free(th);
    free(jobs);
    return rc;
}

typedef struct {
    const uint8_t* packed;
    const uint16_t* scales;
    int width, group;
    const int32_t* ids;
    int T;
    float* out;
    uint16_t* out_bf16;
    int t0, step;
} ple_job;

/* ple-w4-shard-reader.js:85-95: byte i>>1, low nibble for even i, two's complement. */
static void* ple_worker(void* arg) {
    ple_job* j = (ple_job*)arg;
    const int width = j->width;
    const size_t prow = (size_t)width / 2, srow = (size_t)width / j->group;
    for (int t = j->t0; t < j->T; t += j->step) {
        const uint8_t* p = j->packed + (size_t)j->ids[t] * prow;
        const uint16_t* s = j->scales + (size_t)j->ids[t] * srow;
        for (int i = 0; i < width; ++i) {
            const uint32_t byte = p[i >> 1];
            const uint32_t nibble = (i & 1) == 0 ? (byte & 0x0fu) : (byte >> 4);
            const int q = nibble >= 8 ? (int)nibble - 16 : (int)nibble;
            const float scale = g4o_bf16_bits_to_f32(s[i / j->group]);
            const float v = (float)q * scale;
            if (j->out) j->out[(size_t)t * width + i] = v;
            if (j->out_bf16) j->out_bf16[(size_t)t * width + i] = g4o_f32_to_bf16_bits(v);
        }
    }
    return NULL;
}

static int ple_run(const uint8_t* packed, const uint16_t* scales, int vocab, int width, int group,
                   const int32_t* ids, int T, float* out, uint16_t* out_bf16, int nthreads) {
    if (width % 2 != 0 || group <= 0 || width % group != 0) return -1;
    for (int t = 0; t < T; ++t)
        if (ids[t] < 0 || ids[t] >= vocab) return -2; /* ple-w4-shard-reader.js:50-54 */
    if (nthreads < 1) nthreads = 1;
    ple_job base = {packed, scales, width, group, ids, T, out, out_bf16, 0, nthreads};
    if (nthreads == 1) {
        ple_worker(&base);
        return 0;
    }
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
    ple_job* jobs = (ple_job*)malloc(sizeof(ple_job) * nthreads);
    for (int i = 0; i < nthreads; ++i) {
        jobs[i] = base;
        jobs[i].t0 = i;
        pthread_create(&th[i], NULL, ple_worker, &jobs[i]);
    }
    for (int i = 0; i < nthreads; ++i) pthread_join(th[i], NULL);
    free(th);
    free(jobs);
    return 0;
}

int g4o_ple_read_rows(const uint8_t* packed, const uint16_t* scales_bf16, int vocab, int width,
                      int group, const int32_t* ids, int T, float* out, int nthreads) {
    return ple_run(packed, scales_bf16, vocab, width, group, ids, T, out, NULL, nthreads);
}

int g4o_ple_read_rows_bf16(const uint8_t* packed, const uint16_t* scales_bf16, int vocab,
                           int width, int group, const int32_t* ids, int T, uint16_t* out,
                           int nthreads) {
    return ple_run(packed, scales_bf16, vocab, width, group, ids, T, NULL, out, nthreads);
}

/* QK_SHADER (gpu-runtime.js:1204-1221): valid = key <= qp && (!sliding || key + window > qp),
 * masked logits -1e30; SOFTMAX_SHADER (:1223-1234): max, sum of exp, exp/sum;
 * ATTN_OUT_SHADER (:1236-1248): probs . V.  Scale 1.0, one KV head shared by all heads
 * (repeatKVHeads, official-w4a16-layer0.js:16-28). */
int g4o_attention(const float* q, const float* kc, const float* vc, int rows, int heads, int hd,
                  int keylen, int qpos0, int sliding, int window, float* out) {
    if (rows < 0 || heads <= 0 || hd <= 0 || keylen <= 0) return -1;
    float* logits = (float*)malloc(sizeof(float) * (size_t)keylen);
    if (!logits) return -3;
    for (int r = 0; r < rows; ++r) {
        const int qp = qpos0 + r;
        for (int h = 0; h < heads; ++h) {
            const float* qv = q + ((size_t)r * heads + h) * hd;
            for (int key = 0; key < keylen; ++key) {
                int valid = key <= qp;
                if (sliding) valid = valid && (key + window) > qp;
                if (!valid) {
                    logits[key] = -1e30f;
                    continue;
                }
                const float* kv = kc + (size_t)key * hd;
                float acc = 0.f;
                for (int d = 0; d < hd; ++d) acc += qv[d] * kv[d];
                logits[key] = acc;
            }
            float mx = -3.4e38f;
            for (int key = 0; key < keylen; ++key) mx = logits[key] > mx ? logits[key] : mx;
            float ss = 0.f;
            for (int key = 0; key < keylen; ++key) ss += expf(logits[key] - mx);
            for (int key = 0; key < keylen; ++key) logits[key] = expf(logits[key] - mx) / ss;
            float* o = out + ((size_t)r * heads + h) * hd;
            for (int d = 0; d < hd; ++d) {
                float acc = 0.f;
                for (int key = 0; key < keylen; ++key) acc += logits[key] * vc[(size_t)key * hd + d];
                o[d] = acc;
            }
        }
    }
    free(logits);
    return 0;
}
