"""Host-side mirror of the reference's GPU operator API over the g4w4 C ABI.

The reference model graph (custom-webgpu/gemma4-webgpu.js) talks to its runtime
through `GPUOps` (custom-webgpu/gpu-runtime.js:1295-1378), `GPUW4Linear.load`
(:1385-1392), `reader.pleRowsToGpu(device, ids)` (:905, :993, :1050) and `KVCache`
(gemma4-webgpu.js:122-137).  This module exposes the same operators with the same
argument meaning and the same errors (raised as G4Error), over libg4w4.so.
Device buffers are torch CUDA tensors; like the reference, each operator returns
a newly allocated output.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from ._lib import G4_BF16, G4_F32, G4Error, call

_DT = {torch.float32: G4_F32, torch.bfloat16: G4_BF16}


def _ptr(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


def _host_or_device(a) -> tuple[C.c_void_p, int, object]:
    """(pointer, on_device, keepalive) for a numpy array or a contiguous torch tensor."""
    if isinstance(a, torch.Tensor):
        a = a.contiguous()
        return C.c_void_p(a.data_ptr()), int(a.is_cuda), a
    a = np.ascontiguousarray(a)
    return C.c_void_p(a.ctypes.data), 0, a


class Context:
    """One g4_ctx per GPU (the reference's WebGPU device + queue)."""

    def __init__(self, device: int = 0, stream: torch.cuda.Stream | None = None):
        _lib.load()
        self.device = device
        self.torch_device = torch.device("cuda", device)
        s = stream if stream is not None else torch.cuda.current_stream(self.torch_device)
        self._stream = s
        h = C.c_void_p()
        call("g4_ctx_create", device, C.c_void_p(s.cuda_stream), C.byref(h))
        self.handle = h

    def set_stream(self, stream: torch.cuda.Stream) -> None:
        self._stream = stream
        call("g4_ctx_set_stream", self.handle, C.c_void_p(stream.cuda_stream))

    def set_pdl(self, enable: bool) -> None:
        """Programmatic dependent launch for this context's kernels (g4_ctx_set_pdl)."""
        call("g4_ctx_set_pdl", self.handle, int(bool(enable)))

    @property
    def stream(self) -> torch.cuda.Stream:
        return self._stream

    def sync(self) -> None:
        call("g4_stream_sync", self.handle)

    def check_device(self) -> int:
        """Raises G4Error if a kernel raised the device error word since the last check."""
        flags = C.c_uint32(0)
        st = _lib.load().g4_ctx_check_device(self.handle, C.byref(flags))
        _lib.check(st)
        return flags.value

    def close(self) -> None:
        if getattr(self, "handle", None):
            _lib.load().g4_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class W4Linear:
    """GPUW4Linear (gpu-runtime.js:1380-1394): packed int32 [N, K/8] + bf16 scales [N, K/group]."""

    def __init__(self, ctx: Context, packed, scales, group_size: int = 32, name: str = ""):
        self.ctx = ctx
        self.name = name
        out_dim = int(packed.shape[0])
        in_dim = int(packed.shape[1]) * 8
        groups = int(scales.shape[1])
        if groups == 0 or in_dim % groups:
            raise G4Error(-1, f"{name}: scale shape {tuple(scales.shape)} does not divide K={in_dim}")
        group_size = in_dim // groups  # gpu-runtime.js:1388 derives it from the shapes
        if isinstance(scales, torch.Tensor) and scales.dtype == torch.bfloat16:
            scales = scales.view(torch.int16)
        pp, pd, keep1 = _host_or_device(packed)
        sp, sd, keep2 = _host_or_device(scales)
        if pd != sd:
            raise G4Error(-1, "packed and scales must both be on the host or both on the device")
        h = C.c_void_p()
        call("g4_linear_create", ctx.handle, pp, sp, in_dim, out_dim, group_size, pd, C.byref(h))
        self.handle = h
        self.in_dim, self.out_dim, self.group_size, self.groups = in_dim, out_dim, group_size, groups

    def dequant(self, row_start: int = 0, row_count: int | None = None, dtype=torch.float32) -> torch.Tensor:
        rc = self.out_dim - row_start if row_count is None else row_count
        out = torch.empty((rc, self.in_dim), dtype=dtype, device=self.ctx.torch_device)
        call("g4_linear_dequant", self.ctx.handle, self.handle, row_start, rc, _ptr(out), _DT[dtype])
        return out

    def close(self):
        if getattr(self, "handle", None):
            _lib.load().g4_linear_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PleW4Table:
    """Device-resident PLE W4 table; rows_to_gpu mirrors reader.pleRowsToGpu(device, ids)."""

    def __init__(self, ctx: Context, packed, scales, vocab: int | None = None, width: int = 8960, group: int = 32):
        self.ctx = ctx
        if packed is None:
            assert vocab is not None
            h = C.c_void_p()
            call("g4_ple_table_create", ctx.handle, None, None, vocab, width, group, 0, C.byref(h))
        else:
            vocab = int(packed.shape[0])
            width = int(packed.shape[1]) * 2
            if isinstance(scales, torch.Tensor) and scales.dtype == torch.bfloat16:
                scales = scales.view(torch.int16)
            pp, pd, k1 = _host_or_device(packed)
            sp, sd, k2 = _host_or_device(scales)
            h = C.c_void_p()
            call("g4_ple_table_create", ctx.handle, pp, sp, vocab, width, group, pd, C.byref(h))
        self.handle = h
        self.vocab, self.width, self.group = vocab, width, group

    def upload_rows(self, row_start: int, packed, scales) -> None:
        pp, pd, k1 = _host_or_device(packed)
        sp, sd, k2 = _host_or_device(scales)
        call("g4_ple_table_upload_rows", self.ctx.handle, self.handle, row_start, int(packed.shape[0]), pp, sp, pd)
        if pd:
            self.ctx.sync()

    def rows_to_gpu(self, ids, dtype=torch.float32, out: torch.Tensor | None = None) -> torch.Tensor:
        """[T, width] dequantised rows (f32 like the reference, or bf16)."""
        if isinstance(ids, torch.Tensor) and ids.is_cuda:
            ids_t = ids.to(torch.int32).contiguous()
            T, ptr, on_dev, keep = ids_t.numel(), _ptr(ids_t), 1, ids_t
        else:
            arr = np.ascontiguousarray(np.asarray(ids, dtype=np.int64))
            if arr.size and (arr.min() < -(2**31) or arr.max() >= 2**31):
                raise G4Error(-6, f"PLE token id out of range: {int(arr.max())}")
            keep = arr.astype(np.int32)
            T, ptr, on_dev = keep.size, C.c_void_p(keep.ctypes.data), 0
        if out is None:
            out = torch.empty((T, self.width), dtype=dtype, device=self.ctx.torch_device)
        call("g4_ple_gather", self.ctx.handle, self.handle, ptr, T, on_dev, _ptr(out), _DT[out.dtype])
        return out

    def close(self):
        if getattr(self, "handle", None):
            _lib.load().g4_ple_table_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KVCache:
    """KVCache (gemma4-webgpu.js:122-137) with bf16 storage.

    ring > 0: a sliding-window cache of `nseq` sequences that keeps each sequence's last
    `ring` positions (g4_kv_create_ring); max_seq stays the position limit.  `rows` is the
    storage height and `seq_rows` the row stride per sequence."""

    def __init__(self, ctx: Context, head_dim: int, max_seq: int, ring: int = 0, nseq: int = 1):
        self.ctx = ctx
        h = C.c_void_p()
        if ring:
            call("g4_kv_create_ring", ctx.handle, head_dim, max_seq, ring, nseq, C.byref(h))
        else:
            call("g4_kv_create", ctx.handle, head_dim, max_seq, C.byref(h))
        self.handle = h
        self.head_dim, self.max_seq = head_dim, max_seq
        r, sr, n = C.c_int(0), C.c_int(0), C.c_int(0)
        call("g4_kv_layout", h, C.byref(r), C.byref(sr), C.byref(n))
        self.ring, self.seq_rows, self.nseq = r.value, sr.value, n.value
        self.rows = self.seq_rows * self.nseq if self.ring else max_seq

    def slot(self, pos: int) -> int:
        """Storage row of position pos (of sequence 0)."""
        return pos % self.ring if self.ring else pos

    @property
    def length(self) -> int:
        n = C.c_int(0)
        call("g4_kv_info", self.handle, C.byref(n), None, None)
        return n.value

    def append(self, k: torch.Tensor, v: torch.Tensor, rows: int, start_pos: int) -> None:
        k = k.contiguous()
        v = v.contiguous()
        if k.dtype != v.dtype or k.dtype not in _DT:
            raise G4Error(-1, "KV append wants f32 or bf16 k and v of one dtype")
        call("g4_kv_append", self.ctx.handle, self.handle, _ptr(k), _ptr(v), rows, start_pos, _DT[k.dtype])

    def reset(self) -> None:
        call("g4_kv_reset", self.handle)

    def tensors(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Copies of the bf16 K and V storage [rows, head_dim] (for tests)."""
        kp, vp = C.c_void_p(), C.c_void_p()
        call("g4_kv_buffers", self.handle, C.byref(kp), C.byref(vp))
        n = self.rows * self.head_dim
        return _wrap_device(kp.value, n, self.ctx).view(self.rows, self.head_dim), \
            _wrap_device(vp.value, n, self.ctx).view(self.rows, self.head_dim)

    def close(self):
        if getattr(self, "handle", None):
            _lib.load().g4_kv_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _wrap_device(ptr: int, n: int, ctx: Context) -> torch.Tensor:
    """Copies n bf16 values from a library-owned device pointer into a new tensor."""
    out = torch.empty(n, dtype=torch.bfloat16, device=ctx.torch_device)
    ctx.sync()
    cudart = C.CDLL("libcudart.so.12")
    cudart.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    res = cudart.cudaMemcpy(C.c_void_p(out.data_ptr()), C.c_void_p(ptr), n * 2, 3)  # device to device
    if int(res) != 0:
        raise G4Error(-3, f"cudaMemcpy failed ({res})")
    return out


class GPUOps:
    """GPUOps (gpu-runtime.js:1295-1378) over libg4w4, method for method.

    Every operator takes and returns the reference's f32 buffers (a new output per call,
    like `emptyF32`); w4 and attention also take bf16 activations (the W4A16 kernels'
    own input type), returning bf16 unless asked otherwise."""

    def __init__(self, ctx: Context):
        self.ctx = ctx

    def _f32(self, n: int) -> torch.Tensor:
        return torch.empty(n, dtype=torch.float32, device=self.ctx.torch_device)

    @staticmethod
    def _need_f32(name: str, *ts: torch.Tensor) -> None:
        for t in ts:
            if t.dtype != torch.float32:
                raise G4Error(-1, f"{name}: f32 buffers expected, got {t.dtype}")

    def w4(self, linear: W4Linear, x: torch.Tensor, rows: int, out_dtype=None, impl: int = 0,
           out: torch.Tensor | None = None) -> torch.Tensor:
        """GPUOps.w4(encoder, linear, x, rows): y[rows, outDim] = x . dequant(W)^T.  f32 x (the
        reference's buffers) gives f32 y through g4_linear_w4a16_f32; bf16 x runs the kernels
        directly (bf16 out unless out_dtype / out say f32)."""
        x = x.contiguous()
        if x.numel() != rows * linear.in_dim:
            raise G4Error(-1, f"{linear.name}: x has {x.numel()} values, expected {rows}x{linear.in_dim}")
        if x.dtype == torch.float32:
            if impl != 0 or (out_dtype not in (None, torch.float32)):
                raise G4Error(-1, f"{linear.name}: f32 x gives f32 y through the automatic kernel choice")
            if out is None:
                out = torch.empty((rows, linear.out_dim), dtype=torch.float32, device=self.ctx.torch_device)
            call("g4_linear_w4a16_f32", self.ctx.handle, linear.handle, _ptr(x), rows, _ptr(out))
            return out
        if x.dtype != torch.bfloat16:
            raise G4Error(-1, f"{linear.name}: x must be f32 or bf16, got {x.dtype}")
        if out is None:
            out = torch.empty((rows, linear.out_dim), dtype=out_dtype or torch.bfloat16, device=self.ctx.torch_device)
        call("g4_linear_w4a16_impl", self.ctx.handle, linear.handle, _ptr(x), rows, _ptr(out), _DT[out.dtype], impl)
        return out

    def rms(self, x: torch.Tensor, rows: int, width: int, scale: torch.Tensor | None = None) -> torch.Tensor:
        """GPUOps.rms(encoder, x, rows, width, scale) (RMS_SHADER, eps 1e-6)."""
        self._need_f32("rms", x, *([scale] if scale is not None else []))
        y = self._f32(rows * width)
        call("g4_rms", self.ctx.handle, _ptr(x), _ptr(scale) if scale is not None else None, rows, width,
             C.c_float(1e-6), _ptr(y), G4_F32)
        return y

    def addScale(self, a: torch.Tensor, b: torch.Tensor, n: int, scale: float = 1.0) -> torch.Tensor:  # noqa: N802
        """GPUOps.addScale(encoder, a, b, n, scale)."""
        self._need_f32("addScale", a, b)
        y = self._f32(n)
        call("g4_add_scale", self.ctx.handle, _ptr(a), _ptr(b), n, C.c_float(scale), _ptr(y))
        return y

    def scale(self, a: torch.Tensor, n: int, s: float) -> torch.Tensor:
        """GPUOps.scale(encoder, a, n, s)."""
        self._need_f32("scale", a)
        y = self._f32(n)
        call("g4_scale", self.ctx.handle, _ptr(a), n, C.c_float(s), _ptr(y))
        return y

    def geluMul(self, gate: torch.Tensor, up: torch.Tensor, n: int) -> torch.Tensor:  # noqa: N802
        """GPUOps.geluMul(encoder, gate, up, n)."""
        self._need_f32("geluMul", gate, up)
        y = self._f32(n)
        call("g4_gelu_mul_f32", self.ctx.handle, _ptr(gate), _ptr(up), n, _ptr(y))
        return y

    def geluPle(self, gate: torch.Tensor, ple: torch.Tensor, rows: int, layer: int,  # noqa: N802
                layers: int = 35, dim: int = 256) -> torch.Tensor:
        """GPUOps.geluPle(encoder, gate, ple, rows, layer): ple is [rows, 35, 256]."""
        self._need_f32("geluPle", gate, ple)
        y = self._f32(rows * dim)
        call("g4_gelu_ple_f32", self.ctx.handle, _ptr(gate), _ptr(ple), rows, layer, layers, dim, _ptr(y))
        return y

    def normRope(self, x: torch.Tensor, rows: int, heads: int, hd: int, pos0: int, scale: torch.Tensor,  # noqa: N802
                 ropeProp: float, base: float) -> torch.Tensor:  # noqa: N803
        """GPUOps.normRope(encoder, x, rows, heads, hd, pos0, scale, ropeProp, base)."""
        self._need_f32("normRope", x, scale)
        y = self._f32(rows * heads * hd)
        call("g4_norm_rope", self.ctx.handle, _ptr(x), rows, heads, hd, pos0, _ptr(scale), int(ropeProp * hd / 2),
             C.c_float(base), C.c_float(1e-6), _ptr(y))
        return y

    def attention(self, q: torch.Tensor, cache: KVCache, qrows: int, heads: int, hd: int, keylen: int,
                  qpos0: int, sliding: bool, window: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """GPUOps.attention(encoder, q, kcache, vcache, qrows, heads, hd, keylen, qpos0, sliding, window):
        the cache object stands for the reference's kcache/vcache pair.  f32 q (the reference's
        buffers) gives an f32 result through g4_attention_f32; bf16 q gives bf16."""
        q = q.contiguous()
        if q.dtype == torch.float32:
            if out is None:
                out = torch.empty((qrows, heads, hd), dtype=torch.float32, device=self.ctx.torch_device)
            call("g4_attention_f32", self.ctx.handle, _ptr(q), cache.handle, qrows, heads, hd, keylen, qpos0,
                 int(bool(sliding)), window, _ptr(out))
            return out
        if q.dtype != torch.bfloat16:
            raise G4Error(-1, f"attention: q must be f32 or bf16, got {q.dtype}")
        if out is None:
            out = torch.empty((qrows, heads, hd), dtype=torch.bfloat16, device=self.ctx.torch_device)
        call("g4_attention", self.ctx.handle, _ptr(q), cache.handle, qrows, heads, hd, keylen, qpos0,
             int(bool(sliding)), window, _ptr(out))
        return out

    def pleMix(self, proj: torch.Tensor, normScale: torch.Tensor, tokenPle: torch.Tensor, rows: int,  # noqa: N802,N803
               layers: int = 35, dim: int = 256) -> torch.Tensor:
        """GPUOps.pleMix(encoder, proj, normScale, tokenPle, rows): the reference scales proj
        beforehand (ops.scale by 1/sqrt(hidden)); proj here is that scaled projection."""
        self._need_f32("pleMix", proj, normScale, tokenPle)
        y = self._f32(rows * layers * dim)
        call("g4_ple_mix", self.ctx.handle, _ptr(proj), C.c_float(1.0), _ptr(normScale), _ptr(tokenPle), rows,
             layers, dim, C.c_float(1e-6), _ptr(y))
        return y


def launch_count() -> int:
    return int(_lib.load().g4_kernel_launch_count())
