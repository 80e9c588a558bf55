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
    """KVCache (gemma4-webgpu.js:122-137) with bf16 storage."""

    def __init__(self, ctx: Context, head_dim: int, max_seq: int):
        self.ctx = ctx
        h = C.c_void_p()
        call("g4_kv_create", ctx.handle, head_dim, max_seq, C.byref(h))
        self.handle = h
        self.head_dim, self.max_seq = head_dim, max_seq

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
        """Copies of the bf16 K and V storage [max_seq, head_dim] (for tests)."""
        kp, vp = C.c_void_p(), C.c_void_p()
        call("g4_kv_buffers", self.handle, C.byref(kp), C.byref(vp))
        n = self.max_seq * self.head_dim
        return _wrap_device(kp.value, n, self.ctx).view(self.max_seq, self.head_dim), \
            _wrap_device(vp.value, n, self.ctx).view(self.max_seq, self.head_dim)

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
    """GPUOps (gpu-runtime.js:1295-1378): w4 and attention over libg4w4."""

    def __init__(self, ctx: Context):
        self.ctx = ctx

    def w4(self, linear: W4Linear, x: torch.Tensor, rows: int, out_dtype=torch.bfloat16, impl: int = 0,
           out: torch.Tensor | None = None) -> torch.Tensor:
        """GPUOps.w4(encoder, linear, x, rows): y[rows, outDim] = x . dequant(W)^T."""
        if x.dtype != torch.bfloat16:
            raise G4Error(-1, f"{linear.name}: x must be bf16 (W4A16), got {x.dtype}")
        x = x.contiguous()
        if x.numel() != rows * linear.in_dim:
            raise G4Error(-1, f"{linear.name}: x has {x.numel()} values, expected {rows}x{linear.in_dim}")
        if out is None:
            out = torch.empty((rows, linear.out_dim), dtype=out_dtype, device=self.ctx.torch_device)
        call("g4_linear_w4a16_impl", self.ctx.handle, linear.handle, _ptr(x), rows, _ptr(out), _DT[out.dtype], impl)
        return out

    def attention(self, q: torch.Tensor, cache: KVCache, qrows: int, heads: int, hd: int, keylen: int,
                  qpos0: int, sliding: bool, window: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """GPUOps.attention(encoder, q, kcache, vcache, qrows, heads, hd, keylen, qpos0, sliding, window)."""
        if q.dtype != torch.bfloat16:
            raise G4Error(-1, "attention: q must be bf16")
        q = q.contiguous()
        if out is None:
            out = torch.empty((qrows, heads, hd), dtype=torch.bfloat16, device=self.ctx.torch_device)
        call("g4_attention", self.ctx.handle, _ptr(q), cache.handle, qrows, heads, hd, keylen, qpos0,
             int(bool(sliding)), window, _ptr(out))
        return out


def launch_count() -> int:
    return int(_lib.load().g4_kernel_launch_count())
