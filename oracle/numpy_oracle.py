"""Vectorised numpy twin of g4_oracle.c (TEST INFRASTRUCTURE ONLY).

Used to cross-check the C restatement and to produce expected values quickly in
tests.  Each function cites the reference lines it restates (gemma4-js paths).
"""
from __future__ import annotations

import numpy as np

from . import bf16_bits_to_f32, f32_to_bf16_bits


def unpack_linear_q(packed: np.ndarray) -> np.ndarray:
    """official-w4a16.js:21-28 + :15-19: word j nibble k -> column 8j+k, value nibble-8."""
    p = np.ascontiguousarray(packed).view(np.uint32)
    N, W = p.shape
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    nib = (p[:, :, None] >> shifts) & 0xF
    return nib.reshape(N, W * 8).astype(np.int8) - 8


def dequant_w4a16(packed: np.ndarray, scales_bf16: np.ndarray, group: int = 32) -> np.ndarray:
    """dequantizeOfficialW4A16Rows (official-w4a16.js:50-101) for all rows, f32."""
    q = unpack_linear_q(packed).astype(np.float32)
    s = bf16_bits_to_f32(scales_bf16)
    return q * np.repeat(s, group, axis=1)


def linear_w4a16(x: np.ndarray, packed: np.ndarray, scales_bf16: np.ndarray, group: int = 32) -> np.ndarray:
    """OfficialW4A16Linear.apply (official-quantized-linear.js:82-128), float64 dot then f32."""
    w = dequant_w4a16(packed, scales_bf16, group).astype(np.float64)
    return (np.asarray(x, np.float64) @ w.T).astype(np.float32)


def ple_unpack_q(packed: np.ndarray) -> np.ndarray:
    """ple-w4-shard-reader.js:89-92: low nibble = even column, two's complement."""
    b = np.asarray(packed, np.uint8)
    lo = (b & 0x0F).astype(np.int16)
    hi = (b >> 4).astype(np.int16)
    q = np.empty(b.shape[:-1] + (b.shape[-1] * 2,), np.int16)
    q[..., 0::2] = lo
    q[..., 1::2] = hi
    return np.where(q >= 8, q - 16, q).astype(np.int8)


def ple_read_rows(packed: np.ndarray, scales_bf16: np.ndarray, ids, group: int = 32, bf16: bool = False):
    """LocalPleW4ShardReader.readRows (ple-w4-shard-reader.js:65-104)."""
    ids = np.asarray(ids, np.int64)
    q = ple_unpack_q(packed[ids]).astype(np.float32)
    s = bf16_bits_to_f32(scales_bf16[ids])
    v = q * np.repeat(s, group, axis=-1)
    return f32_to_bf16_bits(v) if bf16 else v


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, qpos0: int, sliding: bool, window: int,
              keylen: int | None = None) -> np.ndarray:
    """GPUOps.attention (gpu-runtime.js:1204-1248), float64."""
    rows, heads, hd = q.shape
    keylen = k.shape[0] if keylen is None else keylen
    kk = np.asarray(k[:keylen], np.float64)
    vv = np.asarray(v[:keylen], np.float64)
    logits = np.einsum("rhd,kd->rhk", np.asarray(q, np.float64), kk)
    qp = qpos0 + np.arange(rows)[:, None]
    key = np.arange(keylen)[None, :]
    valid = key <= qp
    if sliding:
        valid &= (key + window) > qp
    logits = np.where(valid[:, None, :], logits, -1e30)
    logits -= logits.max(-1, keepdims=True)
    p = np.exp(logits)
    p /= p.sum(-1, keepdims=True)
    return np.einsum("rhk,kd->rhd", p, vv).astype(np.float32)
