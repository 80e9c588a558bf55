// gpu_ops.js -- GPUOps-compatible CUDA runtime for the reference's model graph.
//
// Drop-in for the objects custom-webgpu/gemma4-webgpu.js takes from its WebGPU runtime:
//   GPUOps            custom-webgpu/gpu-runtime.js:1295-1378  -> CudaGPUOps
//   GPUW4Linear.load  :1385-1392                               -> CudaW4Linear.load
//   reader.pleRowsToGpu(device, ids)  :905, :993, :1050        -> CudaPleTable.rowsToGpu(ops, ids)
//   KVCache           gemma4-webgpu.js:122-137                 -> CudaKVCache
// Same method names, argument order and f32 buffer convention: every operator allocates and
// returns a new f32 buffer and pushes its temporaries on `garbage`; `encoder` is accepted and
// ignored (work runs in issue order on the context's CUDA stream, as WebGPU queue order does).
// Buffers are CudaBuffer objects ({ptr: BigInt device pointer, bytes}); destroy() frees them.
import { createRequire } from "node:module";

const require = createRequire(import.meta.url);
const g4 = require("./build/Release/g4w4.node");

const F32 = 0;
const BF16 = 1;

export class CudaBuffer {
  constructor(bytes, label = "") {
    this.bytes = bytes;
    this.label = label;
    this.ptr = g4.alloc(bytes);
  }
  destroy() {
    if (this.ptr !== null) g4.free(this.ptr);
    this.ptr = null;
  }
  at(byteOffset) { return this.ptr + BigInt(byteOffset); }
}

export class CudaGPUOps {
  constructor(device = 0) {
    this.ctx = g4.ctxCreate(device);
  }
  track(garbage, buffer) { if (garbage) garbage.push(buffer); return buffer; }
  emptyF32(n, label = "") { return new CudaBuffer(n * 4, label); }
  upload(typedArray, label = "") {
    const b = new CudaBuffer(typedArray.byteLength, label);
    g4.upload(b.ptr, typedArray);
    return b;
  }
  async readF32(buffer, n) {
    const out = new Float32Array(n);
    g4.download(buffer.ptr, out);
    return out;
  }
  submit() { g4.sync(this.ctx); }

  w4(encoder, linear, x, rows, garbage = null) {
    const y = this.emptyF32(rows * linear.outDim, `${linear.name}:out`);
    g4.w4(this.ctx, linear.handle, x.ptr, rows, y.ptr);
    return y;
  }
  rms(encoder, x, rows, width, scale = null, garbage = null) {
    const y = this.emptyF32(rows * width, "rms-out");
    g4.rms(this.ctx, x.ptr, scale ? scale.ptr : null, rows, width, 1e-6, y.ptr);
    return y;
  }
  addScale(encoder, a, b, n, scale = 1, garbage = null) {
    const y = this.emptyF32(n, "add-out");
    g4.addScale(this.ctx, a.ptr, b.ptr, n, scale, y.ptr);
    return y;
  }
  scale(encoder, a, n, s, garbage = null) {
    const y = this.emptyF32(n, "scale-out");
    g4.scale(this.ctx, a.ptr, n, s, y.ptr);
    return y;
  }
  geluMul(encoder, gate, up, n, garbage = null) {
    const y = this.emptyF32(n, "gelu-mul");
    g4.geluMul(this.ctx, gate.ptr, up.ptr, n, y.ptr);
    return y;
  }
  geluPle(encoder, gate, ple, rows, layer, garbage = null) {
    const y = this.emptyF32(rows * 256, "gelu-ple");
    g4.geluPle(this.ctx, gate.ptr, ple.ptr, rows, layer, 35, 256, y.ptr);
    return y;
  }
  normRope(encoder, x, rows, heads, hd, pos0, scale, ropeProp, base, garbage = null) {
    const y = this.emptyF32(rows * heads * hd, "rope-out");
    g4.normRope(this.ctx, x.ptr, rows, heads, hd, pos0, scale.ptr, Math.floor(ropeProp * hd / 2), base, 1e-6, y.ptr);
    return y;
  }
  // kcache is a CudaKVCache (it holds K and V); vcache is accepted for the reference's argument order.
  attention(encoder, q, kcache, vcache, qrows, heads, hd, keylen, qpos0, sliding, window, garbage = null) {
    const out = this.emptyF32(qrows * heads * hd, "attn-out");
    g4.attention(this.ctx, q.ptr, kcache.handle, qrows, heads, hd, keylen, qpos0, !!sliding, window, out.ptr);
    return out;
  }
  // proj is already scaled by the caller (ops.scale before ops.pleMix, gemma4-webgpu.js:318-321).
  pleMix(encoder, proj, normScale, tokenPle, rows, garbage = null) {
    const y = this.emptyF32(rows * 35 * 256, "ple-mix");
    g4.pleMix(this.ctx, proj.ptr, 1.0, normScale.ptr, tokenPle.ptr, rows, 35, 256, 1e-6, y.ptr);
    return y;
  }
  // One chunk of the tied bf16 head (BF16_HEAD_SHADER): out[outOffset + r] = softcap(x . w_r)
  // for the `rows` vocabulary rows of weightChunk (a CudaDense); x is the f32 [1536] row.
  headChunk(encoder, x, weightChunk, out, outOffset, rows, garbage = null) {
    const xb = this.track(garbage, new CudaBuffer(weightChunk.inDim * 2, "head-x-bf16"));
    g4.convert(this.ctx, x.ptr, F32, xb.ptr, BF16, weightChunk.inDim);
    g4.denseMatmul(this.ctx, weightChunk.handle, xb.ptr, 1, out.at(outOffset * 4));
    g4.softcap(this.ctx, out.at(outOffset * 4), rows, 30.0);
  }
  dispose() { g4.ctxDestroy(this.ctx); }
}

export class CudaW4Linear {
  constructor(ops, name, inDim, outDim, groupSize, handle) {
    Object.assign(this, { ops, name, inDim, outDim, groupSize, handle });
    this.groups = inDim / groupSize;
  }
  // GPUW4Linear.load: outDim/inDim/groupSize derived from the tensor shapes (gpu-runtime.js:1388).
  static async load(ops, reader, base) {
    const pi = reader.info(`${base}.weight_packed`), si = reader.info(`${base}.weight_scale`);
    const outDim = pi.shape[0], inDim = pi.shape[1] * 8, groups = si.shape[1], groupSize = inDim / groups;
    const [pb, sb] = await Promise.all([reader.bytes(`${base}.weight_packed`), reader.bytes(`${base}.weight_scale`)]);
    const packed = new Int32Array(pb.buffer ?? pb, pb.byteOffset ?? 0, outDim * inDim / 8);
    const scales = new Uint16Array(sb.buffer ?? sb, sb.byteOffset ?? 0, outDim * groups);
    return new CudaW4Linear(ops, base, inDim, outDim, groupSize,
                            g4.linearCreate(ops.ctx, packed, scales, inDim, outDim, groupSize));
  }
  dispose() { g4.linearDestroy(this.handle); }
}

export class CudaDense {
  // The tied bf16 embedding (or one chunk of it) as the LM head: w is a Uint16Array [N, K].
  constructor(ops, w, inDim, outDim) {
    Object.assign(this, { ops, inDim, outDim });
    this.handle = g4.denseCreate(ops.ctx, w, inDim, outDim);
  }
  dispose() { g4.denseDestroy(this.handle); }
}

export class CudaKVCache {
  // KVCache: per-layer K and V of [maxSeq, hd], bf16 on the device; append takes the
  // reference's f32 rows and throws its errors (gemma4-webgpu.js:128-135).
  constructor(ops, hd, maxSeq) {
    Object.assign(this, { ops, hd, maxSeq });
    this.handle = g4.kvCreate(ops.ctx, hd, maxSeq);
  }
  get length() { return g4.kvLength(this.handle); }
  append(encoder, k, v, rows, startPos) { g4.kvAppend(this.ops.ctx, this.handle, k.ptr, v.ptr, rows, startPos, F32); }
  reset() { g4.kvReset(this.handle); }
  dispose() { g4.kvDestroy(this.handle); }
}

export class CudaPleTable {
  // The whole [vocab, 8960] W4 table resident on the device, uploaded shard by shard from the
  // gemma4-ple-w4-sharded-v1 files (packed block then scale block per shard).
  constructor(ops, vocab, width = 8960, group = 32) {
    Object.assign(this, { ops, vocab, width, group });
    this.handle = g4.pleTableCreate(ops.ctx, vocab, width, group);
  }
  uploadShard(rowStart, rows, packed, scales) {
    g4.pleTableUploadRows(this.ops.ctx, this.handle, rowStart, rows, packed, scales);
  }
  // reader.pleRowsToGpu(device, ids): f32 [ids.length, width]; throws on an out-of-range id.
  rowsToGpu(ops, ids) {
    const out = ops.emptyF32(ids.length * this.width, "ple-rows");
    g4.pleRows(ops.ctx, this.handle, Int32Array.from(ids), out.ptr, F32);
    return out;
  }
  dispose() { g4.pleTableDestroy(this.handle); }
}
