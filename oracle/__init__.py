"""CPU oracle of the gemma4-js W4A16 hot path.

TEST INFRASTRUCTURE ONLY.  tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference arm use it as the checker and the timed CPU baseline; the
product (libg4w4.so and the gemma4-js_b200 package) never imports it.

`lib()` builds (if needed) and loads liboracle.so, the C restatement in g4_oracle.c;
numpy_oracle.py is a vectorised twin used to cross-check it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "g4_oracle.c"
LIB = HERE / "liboracle.so"
GCC_FLAGS = ["-O3", "-fPIC", "-shared", "-pthread", "-std=c11", "-fno-fast-math", "-ffp-contract=off"]

_lib = None


def build(out: Path = LIB, march: str = "x86-64-v2") -> Path:
    """Compiles g4_oracle.c.  The default target is portable so the file can travel to
    another host; bench.py builds a -march=native copy for timing."""
    if out.exists() and out.stat().st_mtime >= max(SRC.stat().st_mtime, (HERE / "g4_oracle.h").stat().st_mtime):
        return out
    out.parent.mkdir(parents=True, exist_ok=True)
    tmp = str(out) + f".{os.getpid()}.tmp"
    subprocess.run(["gcc", *GCC_FLAGS, f"-march={march}", str(SRC), "-o", tmp, "-lm"], check=True)
    os.replace(tmp, out)
    return out


def lib(path: Path | None = None) -> C.CDLL:
    global _lib
    if path is None and _lib is not None:
        return _lib
    p = build() if path is None else path
    L = C.CDLL(str(p))
    f32p = np.ctypeslib.ndpointer(np.float32, flags="C")
    i32p = np.ctypeslib.ndpointer(np.int32, flags="C")
    u16p = np.ctypeslib.ndpointer(np.uint16, flags="C")
    u8p = np.ctypeslib.ndpointer(np.uint8, flags="C")
    I = C.c_int
    L.g4o_f32_to_bf16_bits.restype = C.c_uint16
    L.g4o_f32_to_bf16_bits.argtypes = [C.c_float]
    L.g4o_dequant_w4a16_rows.restype = I
    L.g4o_dequant_w4a16_rows.argtypes = [i32p, u16p, I, I, I, I, I, f32p]
    L.g4o_dequant_w4a16_par.restype = I
    L.g4o_dequant_w4a16_par.argtypes = [i32p, u16p, I, I, I, f32p, I]
    L.g4o_linear_w4a16.restype = I
    L.g4o_linear_w4a16.argtypes = [f32p, I, i32p, u16p, I, I, I, f32p, I]
    L.g4o_ple_read_rows.restype = I
    L.g4o_ple_read_rows.argtypes = [u8p, u16p, I, I, I, i32p, I, f32p, I]
    L.g4o_ple_read_rows_bf16.restype = I
    L.g4o_ple_read_rows_bf16.argtypes = [u8p, u16p, I, I, I, i32p, I, u16p, I]
    L.g4o_attention.restype = I
    L.g4o_attention.argtypes = [f32p, f32p, f32p, I, I, I, I, I, I, I, f32p]
    if path is None:
        _lib = L
    return L


class OracleError(RuntimeError):
    pass


def _ok(rc: int, what: str) -> None:
    if rc != 0:
        raise OracleError(f"{what} failed ({rc})")


def dequant_w4a16_rows(packed: np.ndarray, scales_bf16: np.ndarray, row_start: int = 0,
                       row_count: int | None = None, group: int = 32) -> np.ndarray:
    N, K = packed.shape[0], packed.shape[1] * 8
    rc = N - row_start if row_count is None else row_count
    out = np.empty((rc, K), np.float32)
    _ok(lib().g4o_dequant_w4a16_rows(np.ascontiguousarray(packed, np.int32).reshape(-1),
                                     np.ascontiguousarray(scales_bf16, np.uint16).reshape(-1),
                                     N, K, row_start, rc, group, out.reshape(-1)), "dequant")
    return out


def dequant_w4a16_par(packed: np.ndarray, scales_bf16: np.ndarray, out: np.ndarray | None = None,
                      group: int = 32, nthreads: int = 1, L: C.CDLL | None = None) -> np.ndarray:
    """Every row of a W4A16 weight dequantised to f32 (official-w4a16.js:50-101) on
    nthreads host threads; `out` ([N, K] f32) is reused when given."""
    N, K = packed.shape[0], packed.shape[1] * 8
    if out is None:
        out = np.empty((N, K), np.float32)
    _ok((L or lib()).g4o_dequant_w4a16_par(np.ascontiguousarray(packed, np.int32).reshape(-1),
                                           np.ascontiguousarray(scales_bf16, np.uint16).reshape(-1), N, K, group,
                                           out.reshape(-1), nthreads), "dequant_par")
    return out


def linear_w4a16(x: np.ndarray, packed: np.ndarray, scales_bf16: np.ndarray, group: int = 32,
                 nthreads: int = 1, L: C.CDLL | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    N = packed.shape[0]
    y = np.empty((M, N), np.float32)
    _ok((L or lib()).g4o_linear_w4a16(x.reshape(-1), M, np.ascontiguousarray(packed, np.int32).reshape(-1),
                                      np.ascontiguousarray(scales_bf16, np.uint16).reshape(-1), K, N, group,
                                      y.reshape(-1), nthreads), "linear")
    return y


def ple_read_rows(packed: np.ndarray, scales_bf16: np.ndarray, ids, group: int = 32, bf16: bool = False,
                  nthreads: int = 1, L: C.CDLL | None = None) -> np.ndarray:
    vocab, width = packed.shape[0], packed.shape[1] * 2
    ids = np.ascontiguousarray(ids, np.int32)
    T = ids.size
    p = np.ascontiguousarray(packed, np.uint8).reshape(-1)
    s = np.ascontiguousarray(scales_bf16, np.uint16).reshape(-1)
    if bf16:
        out = np.empty((T, width), np.uint16)
        rc = (L or lib()).g4o_ple_read_rows_bf16(p, s, vocab, width, group, ids, T, out.reshape(-1), nthreads)
    else:
        out = np.empty((T, width), np.float32)
        rc = (L or lib()).g4o_ple_read_rows(p, s, vocab, width, group, ids, T, out.reshape(-1), nthreads)
    if rc == -2:
        raise OracleError("PLE token out of range")
    _ok(rc, "ple_read_rows")
    return out


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, qpos0: int, sliding: bool, window: int,
              keylen: int | None = None) -> np.ndarray:
    q = np.ascontiguousarray(q, np.float32)
    rows, heads, hd = q.shape
    keylen = k.shape[0] if keylen is None else keylen
    out = np.empty_like(q)
    _ok(lib().g4o_attention(q.reshape(-1), np.ascontiguousarray(k, np.float32).reshape(-1),
                            np.ascontiguousarray(v, np.float32).reshape(-1), rows, heads, hd, keylen, qpos0,
                            int(sliding), window, out.reshape(-1)), "attention")
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """roundFloat32ToBF16 (official-w4a16.js:34-48) on an array: bits + 0x7fff + lsb, >> 16."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)
