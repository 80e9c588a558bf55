/*
 * g4w4_napi.c -- Node-API addon exposing libg4w4.so to the reference's JavaScript runtime.
 *
 * The reference's model graph (custom-webgpu/gemma4-webgpu.js) calls its GPU runtime through
 * GPUOps (custom-webgpu/gpu-runtime.js:1295-1378), GPUW4Linear.load (:1385-1392),
 * reader.pleRowsToGpu (:905, :993, :1050) and KVCache (gemma4-webgpu.js:122-137).  This
 * addon binds the C ABI of include/g4w4.h one function per entry point; gpu_ops.js builds
 * GPUOps-compatible objects on top of it, so the graph keeps calling ops.w4(...),
 * ops.attention(...) and the rest unchanged.
 *
 * Conventions at the JS boundary
 *   - Device pointers and library handles are BigInt (uint64); null / undefined is NULL.
 *   - Host arrays (weights, token ids) are TypedArrays, passed by pointer and length.
 *   - Every g4_* failure throws an Error whose message is g4_last_error_string() (the
 *     reference's `throw new Error(...)` text) and whose code is the status name.
 *   - Device memory for outputs comes from alloc()/free() (cudaMalloc/cudaFree): the
 *     reference's operators allocate their outputs, and gpu_ops.js keeps that.
 *
 * Build (node-gyp, binding.gyp beside this file): links libg4w4.so and libcudart.
 */
#include <node_api.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "g4w4.h"

#define G4N_MAX_ARGS 12

static const char* status_name(g4_status st) {
    switch (st) {
        case G4_ERR_INVALID: return "G4_ERR_INVALID";
        case G4_ERR_OOM: return "G4_ERR_OOM";
        case G4_ERR_CUDA: return "G4_ERR_CUDA";
        case G4_ERR_TIMEOUT: return "G4_ERR_TIMEOUT";
        case G4_ERR_UNSUPPORTED: return "G4_ERR_UNSUPPORTED";
        case G4_ERR_RANGE: return "G4_ERR_RANGE";
        case G4_ERR_DEVICE: return "G4_ERR_DEVICE";
        default: return "G4_ERR";
    }
}

static napi_value undefined(napi_env env) {
    napi_value u;
    napi_get_undefined(env, &u);
    return u;
}

/* Throws the library's message for a failing status; returns undefined either way. */
static napi_value result(napi_env env, g4_status st) {
    if (st != G4_OK) napi_throw_error(env, status_name(st), g4_last_error_string());
    return undefined(env);
}

static int fail(napi_env env, const char* fn, const char* what) {
    char msg[160];
    snprintf(msg, sizeof msg, "%s: %s", fn, what);
    napi_throw_error(env, "G4_ERR_INVALID", msg);
    return 0;
}

typedef struct {
    napi_value v[G4N_MAX_ARGS];
    size_t n;
} args_t;

static int get_args(napi_env env, napi_callback_info info, args_t* a, size_t want, const char* fn) {
    a->n = G4N_MAX_ARGS;
    if (napi_get_cb_info(env, info, &a->n, a->v, NULL, NULL) != napi_ok) return fail(env, fn, "bad call");
    if (a->n < want) {
        char msg[96];
        snprintf(msg, sizeof msg, "%zu arguments, %zu expected", a->n, want);
        return fail(env, fn, msg);
    }
    return 1;
}

static int is_nullish(napi_env env, napi_value v) {
    napi_valuetype t;
    if (napi_typeof(env, v, &t) != napi_ok) return 1;
    return t == napi_null || t == napi_undefined;
}

/* BigInt -> pointer (device pointer or library handle); null / undefined -> NULL. */
static int ptr_of(napi_env env, napi_value v, void** out) {
    if (is_nullish(env, v)) {
        *out = NULL;
        return 1;
    }
    uint64_t p = 0;
    bool lossless = false;
    if (napi_get_value_bigint_uint64(env, v, &p, &lossless) != napi_ok || !lossless) return 0;
    *out = (void*)(uintptr_t)p;
    return 1;
}

static int i32_of(napi_env env, napi_value v, int32_t* out) { return napi_get_value_int32(env, v, out) == napi_ok; }
static int i64_of(napi_env env, napi_value v, int64_t* out) { return napi_get_value_int64(env, v, out) == napi_ok; }
static int f32_of(napi_env env, napi_value v, float* out) {
    double d = 0;
    if (napi_get_value_double(env, v, &d) != napi_ok) return 0;
    *out = (float)d;
    return 1;
}
static int bool_of(napi_env env, napi_value v, int* out) {
    bool b = false;
    if (napi_get_value_bool(env, v, &b) != napi_ok) return 0;
    *out = b ? 1 : 0;
    return 1;
}

/* TypedArray -> host pointer and byte length (checked against the expected element type). */
static int host_of(napi_env env, napi_value v, napi_typedarray_type want, void** data, size_t* elems) {
    napi_typedarray_type t;
    napi_value ab;
    size_t off = 0;
    if (napi_get_typedarray_info(env, v, &t, elems, data, &ab, &off) != napi_ok) return 0;
    return t == want;
}

static napi_value bigint_of(napi_env env, const void* p) {
    napi_value v;
    napi_create_bigint_uint64(env, (uint64_t)(uintptr_t)p, &v);
    return v;
}

static napi_value int_of(napi_env env, int64_t i) {
    napi_value v;
    napi_create_int64(env, i, &v);
    return v;
}

/* Shorthands for the argument parsing of each binding. */
#define ARGS(n, fn)                                  \
    args_t a;                                        \
    if (!get_args(env, info, &a, (n), (fn))) return NULL
#define PTR(i, name, fn)                                                    \
    void* name = NULL;                                                      \
    if (!ptr_of(env, a.v[i], &name)) return fail(env, fn, #name " must be a BigInt pointer"), NULL
#define I32(i, name, fn)                                                    \
    int32_t name = 0;                                                       \
    if (!i32_of(env, a.v[i], &name)) return fail(env, fn, #name " must be an integer"), NULL
#define I64(i, name, fn)                                                    \
    int64_t name = 0;                                                       \
    if (!i64_of(env, a.v[i], &name)) return fail(env, fn, #name " must be an integer"), NULL
#define F32(i, name, fn)                                                    \
    float name = 0;                                                         \
    if (!f32_of(env, a.v[i], &name)) return fail(env, fn, #name " must be a number"), NULL
#define BOOL(i, name, fn)                                                   \
    int name = 0;                                                           \
    if (!bool_of(env, a.v[i], &name)) return fail(env, fn, #name " must be a boolean"), NULL

/* ------------------------------------------------------------------ library ---- */

static napi_value Version(napi_env env, napi_callback_info info) {
    (void)info;
    napi_value v;
    napi_create_string_utf8(env, g4_version(), NAPI_AUTO_LENGTH, &v);
    return v;
}

/* ------------------------------------------------------------ context, memory ---- */

/* ctxCreate(device) -> ctx   (new GPUOps(device), gpu-runtime.js:1296) */
static napi_value CtxCreate(napi_env env, napi_callback_info info) {
    ARGS(1, "ctxCreate");
    I32(0, device, "ctxCreate");
    g4_ctx* ctx = NULL;
    g4_status st = g4_ctx_create(device, NULL, &ctx);
    if (st) return result(env, st);
    return bigint_of(env, ctx);
}

static napi_value CtxDestroy(napi_env env, napi_callback_info info) {
    ARGS(1, "ctxDestroy");
    PTR(0, ctx, "ctxDestroy");
    return result(env, g4_ctx_destroy((g4_ctx*)ctx));
}

static napi_value CtxSetPdl(napi_env env, napi_callback_info info) {
    ARGS(2, "ctxSetPdl");
    PTR(0, ctx, "ctxSetPdl");
    BOOL(1, on, "ctxSetPdl");
    return result(env, g4_ctx_set_pdl((g4_ctx*)ctx, on));
}

/* sync(ctx)   (device.queue.onSubmittedWorkDone) */
static napi_value Sync(napi_env env, napi_callback_info info) {
    ARGS(1, "sync");
    PTR(0, ctx, "sync");
    return result(env, g4_stream_sync((g4_ctx*)ctx));
}

static napi_value CheckDevice(napi_env env, napi_callback_info info) {
    ARGS(1, "checkDevice");
    PTR(0, ctx, "checkDevice");
    uint32_t flags = 0;
    g4_status st = g4_ctx_check_device((g4_ctx*)ctx, &flags);
    if (st) return result(env, st);
    return int_of(env, flags);
}

/* alloc(bytes) -> device pointer; free(ptr).  The outputs every GPUOps method allocates. */
static napi_value Alloc(napi_env env, napi_callback_info info) {
    ARGS(1, "alloc");
    I64(0, bytes, "alloc");
    void* p = NULL;
    if (bytes < 0) return fail(env, "alloc", "negative size"), NULL;
    if (bytes > 0 && cudaMalloc(&p, (size_t)bytes) != cudaSuccess) {
        napi_throw_error(env, "G4_ERR_OOM", "alloc: cudaMalloc failed");
        return NULL;
    }
    return bigint_of(env, p);
}

static napi_value Free(napi_env env, napi_callback_info info) {
    ARGS(1, "free");
    PTR(0, p, "free");
    cudaFree(p);
    return undefined(env);
}

/* upload(ptr, typedArray) / download(ptr, typedArray): whole-array copies, synchronous. */
static napi_value Copy(napi_env env, napi_callback_info info, int to_device) {
    const char* fn = to_device ? "upload" : "download";
    ARGS(2, fn);
    PTR(0, dev, fn);
    napi_typedarray_type t;
    size_t n = 0, off = 0;
    void* data = NULL;
    napi_value ab;
    if (napi_get_typedarray_info(env, a.v[1], &t, &n, &data, &ab, &off) != napi_ok)
        return fail(env, fn, "expected a TypedArray"), NULL;
    size_t esize = 1;
    switch (t) {
        case napi_int16_array: case napi_uint16_array: esize = 2; break;
        case napi_int32_array: case napi_uint32_array: case napi_float32_array: esize = 4; break;
        case napi_float64_array: case napi_bigint64_array: case napi_biguint64_array: esize = 8; break;
        default: esize = 1; break;
    }
    cudaError_t e = to_device ? cudaMemcpy(dev, data, n * esize, cudaMemcpyHostToDevice)
                              : cudaMemcpy(data, dev, n * esize, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        napi_throw_error(env, "G4_ERR_CUDA", cudaGetErrorString(e));
        return NULL;
    }
    return undefined(env);
}
static napi_value Upload(napi_env env, napi_callback_info info) { return Copy(env, info, 1); }
static napi_value Download(napi_env env, napi_callback_info info) { return Copy(env, info, 0); }

/* ------------------------------------------------------------- W4A16 linear ---- */

/* linearCreate(ctx, packed:Int32Array, scales:Uint16Array, K, N, group) -> linear
 * (GPUW4Linear.load, gpu-runtime.js:1385-1392: the raw weight_packed / weight_scale bytes). */
static napi_value LinearCreate(napi_env env, napi_callback_info info) {
    ARGS(6, "linearCreate");
    PTR(0, ctx, "linearCreate");
    void *packed = NULL, *scales = NULL;
    size_t np_ = 0, ns = 0;
    if (!host_of(env, a.v[1], napi_int32_array, &packed, &np_)) return fail(env, "linearCreate", "packed must be an Int32Array"), NULL;
    if (!host_of(env, a.v[2], napi_uint16_array, &scales, &ns)) return fail(env, "linearCreate", "scales must be a Uint16Array"), NULL;
    I32(3, K, "linearCreate");
    I32(4, N, "linearCreate");
    I32(5, group, "linearCreate");
    if (K <= 0 || N <= 0 || group <= 0 || np_ != (size_t)N * (size_t)(K / 8) || ns != (size_t)N * (size_t)(K / group))
        return fail(env, "linearCreate", "array lengths do not match K, N, group"), NULL;
    g4_linear* lin = NULL;
    g4_status st = g4_linear_create((g4_ctx*)ctx, packed, scales, K, N, group, 0, &lin);
    if (st) return result(env, st);
    return bigint_of(env, lin);
}

static napi_value LinearDestroy(napi_env env, napi_callback_info info) {
    ARGS(1, "linearDestroy");
    PTR(0, lin, "linearDestroy");
    return result(env, g4_linear_destroy((g4_linear*)lin));
}

/* w4(ctx, linear, x, rows, y): GPUOps.w4 on the reference's f32 buffers (gpu-runtime.js:1316-1324). */
static napi_value W4(napi_env env, napi_callback_info info) {
    ARGS(5, "w4");
    PTR(0, ctx, "w4");
    PTR(1, lin, "w4");
    PTR(2, x, "w4");
    I32(3, rows, "w4");
    PTR(4, y, "w4");
    return result(env, g4_linear_w4a16_f32((g4_ctx*)ctx, (const g4_linear*)lin, (const float*)x, rows, (float*)y));
}

/* w4Bf16(ctx, linear, x_bf16, rows, y, yDtype): the W4A16 kernels on bf16 activations. */
static napi_value W4Bf16(napi_env env, napi_callback_info info) {
    ARGS(6, "w4Bf16");
    PTR(0, ctx, "w4Bf16");
    PTR(1, lin, "w4Bf16");
    PTR(2, x, "w4Bf16");
    I32(3, rows, "w4Bf16");
    PTR(4, y, "w4Bf16");
    I32(5, dt, "w4Bf16");
    return result(env, g4_linear_w4a16((g4_ctx*)ctx, (const g4_linear*)lin, x, rows, y, (g4_dtype)dt));
}

/* ---------------------------------------------------------------- PLE table ---- */

/* pleTableCreate(ctx, vocab, width, group) -> table; rows arrive shard by shard. */
static napi_value PleTableCreate(napi_env env, napi_callback_info info) {
    ARGS(4, "pleTableCreate");
    PTR(0, ctx, "pleTableCreate");
    I32(1, vocab, "pleTableCreate");
    I32(2, width, "pleTableCreate");
    I32(3, group, "pleTableCreate");
    g4_ple_table* t = NULL;
    g4_status st = g4_ple_table_create((g4_ctx*)ctx, NULL, NULL, vocab, width, group, 0, &t);
    if (st) return result(env, st);
    return bigint_of(env, t);
}

/* pleTableUploadRows(ctx, table, rowStart, rows, packed:Uint8Array, scales:Uint16Array):
 * one shard's packed block and scale block (tools/build_ple_w4_full.py:150-154). */
static napi_value PleTableUploadRows(napi_env env, napi_callback_info info) {
    ARGS(6, "pleTableUploadRows");
    PTR(0, ctx, "pleTableUploadRows");
    PTR(1, tab, "pleTableUploadRows");
    I32(2, row0, "pleTableUploadRows");
    I32(3, rows, "pleTableUploadRows");
    void *packed = NULL, *scales = NULL;
    size_t np_ = 0, ns = 0;
    if (!host_of(env, a.v[4], napi_uint8_array, &packed, &np_)) return fail(env, "pleTableUploadRows", "packed must be a Uint8Array"), NULL;
    if (!host_of(env, a.v[5], napi_uint16_array, &scales, &ns)) return fail(env, "pleTableUploadRows", "scales must be a Uint16Array"), NULL;
    (void)np_;
    (void)ns;
    return result(env, g4_ple_table_upload_rows((g4_ctx*)ctx, (g4_ple_table*)tab, row0, rows, packed, scales, 0));
}

static napi_value PleTableDestroy(napi_env env, napi_callback_info info) {
    ARGS(1, "pleTableDestroy");
    PTR(0, tab, "pleTableDestroy");
    return result(env, g4_ple_table_destroy((g4_ple_table*)tab));
}

/* pleRows(ctx, table, ids:Int32Array, out, dtype): reader.pleRowsToGpu(device, ids)
 * (gpu-runtime.js:905, :993, :1050); host ids are range-checked like :466-470. */
static napi_value PleRows(napi_env env, napi_callback_info info) {
    ARGS(5, "pleRows");
    PTR(0, ctx, "pleRows");
    PTR(1, tab, "pleRows");
    void* ids = NULL;
    size_t n = 0;
    if (!host_of(env, a.v[2], napi_int32_array, &ids, &n)) return fail(env, "pleRows", "ids must be an Int32Array"), NULL;
    PTR(3, out, "pleRows");
    I32(4, dt, "pleRows");
    return result(env, g4_ple_gather((g4_ctx*)ctx, (const g4_ple_table*)tab, (const int32_t*)ids, (int)n, 0, out,
                                     (g4_dtype)dt));
}

/* ----------------------------------------------------------------- KV cache ---- */

/* kvCreate(ctx, hd, capacity) -> kv   (new KVCache, gemma4-webgpu.js:122-127) */
static napi_value KvCreate(napi_env env, napi_callback_info info) {
    ARGS(3, "kvCreate");
    PTR(0, ctx, "kvCreate");
    I32(1, hd, "kvCreate");
    I32(2, cap, "kvCreate");
    g4_kv* kv = NULL;
    g4_status st = g4_kv_create((g4_ctx*)ctx, hd, cap, &kv);
    if (st) return result(env, st);
    return bigint_of(env, kv);
}

static napi_value KvDestroy(napi_env env, napi_callback_info info) {
    ARGS(1, "kvDestroy");
    PTR(0, kv, "kvDestroy");
    return result(env, g4_kv_destroy((g4_kv*)kv));
}

/* kvAppend(ctx, kv, k, v, rows, startPos, dtype)   (KVCache.append, gemma4-webgpu.js:128-135) */
static napi_value KvAppend(napi_env env, napi_callback_info info) {
    ARGS(7, "kvAppend");
    PTR(0, ctx, "kvAppend");
    PTR(1, kv, "kvAppend");
    PTR(2, k, "kvAppend");
    PTR(3, v, "kvAppend");
    I32(4, rows, "kvAppend");
    I32(5, start, "kvAppend");
    I32(6, dt, "kvAppend");
    return result(env, g4_kv_append((g4_ctx*)ctx, (g4_kv*)kv, k, v, rows, start, (g4_dtype)dt));
}

/* kvLength(kv) -> length */
static napi_value KvLength(napi_env env, napi_callback_info info) {
    ARGS(1, "kvLength");
    PTR(0, kv, "kvLength");
    int length = 0, hd = 0, cap = 0;
    g4_status st = g4_kv_info((const g4_kv*)kv, &length, &hd, &cap);
    if (st) return result(env, st);
    return int_of(env, length);
}

/* kvReset(kv)   (resetCache, gemma4-webgpu.js:193-196) */
static napi_value KvReset(napi_env env, napi_callback_info info) {
    ARGS(1, "kvReset");
    PTR(0, kv, "kvReset");
    return result(env, g4_kv_reset((g4_kv*)kv));
}

/* attention(ctx, q, kv, rows, heads, hd, keylen, qpos0, sliding, window, out):
 * GPUOps.attention on f32 q and an f32 result (gpu-runtime.js:1357-1365). */
static napi_value Attention(napi_env env, napi_callback_info info) {
    ARGS(11, "attention");
    PTR(0, ctx, "attention");
    PTR(1, q, "attention");
    PTR(2, kv, "attention");
    I32(3, rows, "attention");
    I32(4, heads, "attention");
    I32(5, hd, "attention");
    I32(6, keylen, "attention");
    I32(7, qpos0, "attention");
    BOOL(8, sliding, "attention");
    I32(9, window, "attention");
    PTR(10, out, "attention");
    return result(env, g4_attention_f32((g4_ctx*)ctx, (const float*)q, (const g4_kv*)kv, rows, heads, hd, keylen,
                                        qpos0, sliding, window, (float*)out));
}

/* ------------------------------------------------------- row-wise operators ---- */

/* rms(ctx, x, scale|null, rows, width, eps, out)   (GPUOps.rms, RMS_SHADER :1104-1118) */
static napi_value Rms(napi_env env, napi_callback_info info) {
    ARGS(7, "rms");
    PTR(0, ctx, "rms");
    PTR(1, x, "rms");
    PTR(2, scale, "rms");
    I32(3, rows, "rms");
    I32(4, width, "rms");
    F32(5, eps, "rms");
    PTR(6, out, "rms");
    return result(env, g4_rms((g4_ctx*)ctx, (const float*)x, (const float*)scale, rows, width, eps, out, G4_F32));
}

/* addScale(ctx, a, b, n, scale, y)   (GPUOps.addScale, :1120-1128) */
static napi_value AddScale(napi_env env, napi_callback_info info) {
    ARGS(6, "addScale");
    PTR(0, ctx, "addScale");
    PTR(1, x, "addScale");
    PTR(2, b, "addScale");
    I64(3, n, "addScale");
    F32(4, s, "addScale");
    PTR(5, y, "addScale");
    return result(env, g4_add_scale((g4_ctx*)ctx, (const float*)x, (const float*)b, n, s, (float*)y));
}

/* scale(ctx, a, n, s, y)   (GPUOps.scale, :1130-1137) */
static napi_value Scale(napi_env env, napi_callback_info info) {
    ARGS(5, "scale");
    PTR(0, ctx, "scale");
    PTR(1, x, "scale");
    I64(2, n, "scale");
    F32(3, s, "scale");
    PTR(4, y, "scale");
    return result(env, g4_scale((g4_ctx*)ctx, (const float*)x, n, s, (float*)y));
}

/* geluMul(ctx, gate, up, n, y)   (GPUOps.geluMul, :1139-1157) */
static napi_value GeluMul(napi_env env, napi_callback_info info) {
    ARGS(5, "geluMul");
    PTR(0, ctx, "geluMul");
    PTR(1, gate, "geluMul");
    PTR(2, up, "geluMul");
    I64(3, n, "geluMul");
    PTR(4, y, "geluMul");
    return result(env, g4_gelu_mul_f32((g4_ctx*)ctx, (const float*)gate, (const float*)up, n, (float*)y));
}

/* geluPle(ctx, gate, ple, rows, layer, layers, dim, y)   (GPUOps.geluPle, :1159-1173) */
static napi_value GeluPle(napi_env env, napi_callback_info info) {
    ARGS(8, "geluPle");
    PTR(0, ctx, "geluPle");
    PTR(1, gate, "geluPle");
    PTR(2, ple, "geluPle");
    I32(3, rows, "geluPle");
    I32(4, layer, "geluPle");
    I32(5, layers, "geluPle");
    I32(6, dim, "geluPle");
    PTR(7, y, "geluPle");
    return result(env, g4_gelu_ple_f32((g4_ctx*)ctx, (const float*)gate, (const float*)ple, rows, layer, layers, dim,
                                       (float*)y));
}

/* normRope(ctx, x, rows, heads, hd, pos0, scale, ropeAngles, base, eps, y)   (GPUOps.normRope, :1175-1202) */
static napi_value NormRope(napi_env env, napi_callback_info info) {
    ARGS(11, "normRope");
    PTR(0, ctx, "normRope");
    PTR(1, x, "normRope");
    I32(2, rows, "normRope");
    I32(3, heads, "normRope");
    I32(4, hd, "normRope");
    I32(5, pos0, "normRope");
    PTR(6, scale, "normRope");
    I32(7, angles, "normRope");
    F32(8, base, "normRope");
    F32(9, eps, "normRope");
    PTR(10, y, "normRope");
    return result(env, g4_norm_rope((g4_ctx*)ctx, (const float*)x, rows, heads, hd, pos0, (const float*)scale, angles,
                                    base, eps, (float*)y));
}

/* pleMix(ctx, proj, projScale, norm, tokPle, rows, layers, dim, eps, out)   (GPUOps.pleMix, :1250-1263) */
static napi_value PleMix(napi_env env, napi_callback_info info) {
    ARGS(10, "pleMix");
    PTR(0, ctx, "pleMix");
    PTR(1, proj, "pleMix");
    F32(2, pscale, "pleMix");
    PTR(3, norm, "pleMix");
    PTR(4, tok, "pleMix");
    I32(5, rows, "pleMix");
    I32(6, layers, "pleMix");
    I32(7, dim, "pleMix");
    F32(8, eps, "pleMix");
    PTR(9, out, "pleMix");
    return result(env, g4_ple_mix((g4_ctx*)ctx, (const float*)proj, pscale, (const float*)norm, (const float*)tok, rows,
                                  layers, dim, eps, (float*)out));
}

/* --------------------------------------------------------- tied bf16 head ---- */

/* denseCreate(ctx, w:Uint16Array, K, N) -> dense   (the tied embedding, gemma4-webgpu.js:170-188) */
static napi_value DenseCreate(napi_env env, napi_callback_info info) {
    ARGS(4, "denseCreate");
    PTR(0, ctx, "denseCreate");
    void* w = NULL;
    size_t n = 0;
    if (!host_of(env, a.v[1], napi_uint16_array, &w, &n)) return fail(env, "denseCreate", "w must be a Uint16Array"), NULL;
    I32(2, K, "denseCreate");
    I32(3, N, "denseCreate");
    if (K <= 0 || N <= 0 || n != (size_t)K * (size_t)N) return fail(env, "denseCreate", "w length != K * N"), NULL;
    g4_dense* d = NULL;
    g4_status st = g4_dense_create((g4_ctx*)ctx, w, K, N, 0, &d);
    if (st) return result(env, st);
    return bigint_of(env, d);
}

static napi_value DenseDestroy(napi_env env, napi_callback_info info) {
    ARGS(1, "denseDestroy");
    PTR(0, d, "denseDestroy");
    return result(env, g4_dense_destroy((g4_dense*)d));
}

/* denseMatmul(ctx, dense, x_bf16, M, y)   (BF16_HEAD logits without the softcap, :1265-1277) */
static napi_value DenseMatmul(napi_env env, napi_callback_info info) {
    ARGS(5, "denseMatmul");
    PTR(0, ctx, "denseMatmul");
    PTR(1, d, "denseMatmul");
    PTR(2, x, "denseMatmul");
    I32(3, M, "denseMatmul");
    PTR(4, y, "denseMatmul");
    return result(env, g4_dense_matmul((g4_ctx*)ctx, (const g4_dense*)d, x, M, (float*)y));
}

/* softcap(ctx, logits, n, cap)   (the softcap of BF16_HEAD, in place) */
static napi_value Softcap(napi_env env, napi_callback_info info) {
    ARGS(4, "softcap");
    PTR(0, ctx, "softcap");
    PTR(1, logits, "softcap");
    I64(2, n, "softcap");
    F32(3, cap, "softcap");
    return result(env, g4_softcap((g4_ctx*)ctx, (float*)logits, n, cap));
}

/* softcapArgmax(ctx, logits, rows, vocab, cap, ids, vals|null)   (greedy, gemma4-webgpu.js:465-478) */
static napi_value SoftcapArgmax(napi_env env, napi_callback_info info) {
    ARGS(7, "softcapArgmax");
    PTR(0, ctx, "softcapArgmax");
    PTR(1, logits, "softcapArgmax");
    I32(2, rows, "softcapArgmax");
    I32(3, vocab, "softcapArgmax");
    F32(4, cap, "softcapArgmax");
    PTR(5, ids, "softcapArgmax");
    PTR(6, vals, "softcapArgmax");
    return result(env, g4_softcap_argmax((g4_ctx*)ctx, (const float*)logits, rows, vocab, cap, (int32_t*)ids,
                                         (float*)vals));
}

/* convert(ctx, src, srcDtype, dst, dstDtype, n)   (f32 <-> bf16 with the reference's rounding) */
static napi_value Convert(napi_env env, napi_callback_info info) {
    ARGS(6, "convert");
    PTR(0, ctx, "convert");
    PTR(1, src, "convert");
    I32(2, sdt, "convert");
    PTR(3, dst, "convert");
    I32(4, ddt, "convert");
    I64(5, n, "convert");
    return result(env, g4_convert((g4_ctx*)ctx, src, (g4_dtype)sdt, dst, (g4_dtype)ddt, n));
}

/* ---------------------------------------------------------------- exports ---- */

#define FN(js, c) {js, NULL, c, NULL, NULL, NULL, napi_default, NULL}

NAPI_MODULE_INIT() {
    static const napi_property_descriptor fns[] = {
        FN("version", Version),
        FN("ctxCreate", CtxCreate),
        FN("ctxDestroy", CtxDestroy),
        FN("ctxSetPdl", CtxSetPdl),
        FN("sync", Sync),
        FN("checkDevice", CheckDevice),
        FN("alloc", Alloc),
        FN("free", Free),
        FN("upload", Upload),
        FN("download", Download),
        FN("linearCreate", LinearCreate),
        FN("linearDestroy", LinearDestroy),
        FN("w4", W4),
        FN("w4Bf16", W4Bf16),
        FN("pleTableCreate", PleTableCreate),
        FN("pleTableUploadRows", PleTableUploadRows),
        FN("pleTableDestroy", PleTableDestroy),
        FN("pleRows", PleRows),
        FN("kvCreate", KvCreate),
        FN("kvDestroy", KvDestroy),
        FN("kvAppend", KvAppend),
        FN("kvLength", KvLength),
        FN("kvReset", KvReset),
        FN("attention", Attention),
        FN("rms", Rms),
        FN("addScale", AddScale),
        FN("scale", Scale),
        FN("geluMul", GeluMul),
        FN("geluPle", GeluPle),
        FN("normRope", NormRope),
        FN("pleMix", PleMix),
        FN("denseCreate", DenseCreate),
        FN("denseDestroy", DenseDestroy),
        FN("denseMatmul", DenseMatmul),
        FN("softcap", Softcap),
        FN("softcapArgmax", SoftcapArgmax),
        FN("convert", Convert),
    };
    napi_define_properties(env, exports, sizeof fns / sizeof fns[0], fns);
    return exports;
}
