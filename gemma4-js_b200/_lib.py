"""ctypes binding of libg4w4.so (the C ABI declared in include/g4w4.h).

This is the Python twin of the N-API addon a Node host would load: plain pointers,
sizes and status codes.  There is deliberately no fallback: if the CUDA library is
missing, importing the runtime fails.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libg4w4.so"
HEADER = PKG.parent / "include" / "g4w4.h"

G4_OK = 0
G4_ROWS_HISTORY_READY = 1
G4_F32 = 0
G4_BF16 = 1


class G4Rows(C.Structure):
    """g4_rows: where the rows of a batch sit in their sequences (include/g4w4.h)."""
    _fields_ = [("seq_pos", C.c_void_p), ("seq_base", C.c_int), ("rows_per_seq", C.c_int), ("pos0", C.c_int),
                ("flags", C.c_int)]


class G4Planes(C.Structure):
    """g4_planes: a linear's f32 output as partial planes summed in slice order (include/g4w4.h)."""
    _fields_ = [("base", C.c_void_p), ("count", C.c_int), ("stride", C.c_longlong), ("ld", C.c_int)]

class G4DecoderLayer(C.Structure):
    """g4_decoder_layer (include/g4w4.h)."""
    _fields_ = [("qkv", C.c_void_p), ("o", C.c_void_p), ("gu", C.c_void_p), ("down", C.c_void_p),
                ("pg", C.c_void_p), ("pp", C.c_void_p),
                ("n_in", C.c_void_p), ("n_pa", C.c_void_p), ("n_pf", C.c_void_p), ("n_pff", C.c_void_p),
                ("n_pple", C.c_void_p), ("qn", C.c_void_p), ("kn", C.c_void_p),
                ("skip", C.c_float), ("kv", C.c_void_p), ("has_kv", C.c_int), ("full", C.c_int),
                ("rope_angles", C.c_int), ("rope_base", C.c_float), ("inter", C.c_int)]


class G4DecoderDesc(C.Structure):
    """g4_decoder_desc (include/g4w4.h)."""
    _fields_ = [("layers", C.c_int), ("hidden", C.c_int), ("heads", C.c_int), ("ple_dim", C.c_int),
                ("window", C.c_int), ("vocab", C.c_int), ("eps", C.c_float), ("softcap", C.c_float),
                ("top", C.c_void_p), ("ple_norm", C.c_void_p), ("final_norm", C.c_void_p), ("embed", C.c_void_p),
                ("ple", C.c_void_p)]


STATUS_NAMES = {
    0: "G4_OK", -1: "G4_ERR_INVALID", -2: "G4_ERR_OOM", -3: "G4_ERR_CUDA", -4: "G4_ERR_TIMEOUT",
    -5: "G4_ERR_UNSUPPORTED", -6: "G4_ERR_RANGE", -7: "G4_ERR_DEVICE",
}


class G4Error(RuntimeError):
    """A failing g4w4 call; `.status` is the g4_status code, str() the library message."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status
        self.status_name = STATUS_NAMES.get(status, str(status))


_P = C.c_void_p
_I = C.c_int
_S = C.c_int32
_F = C.c_float
_PP = C.POINTER(C.c_void_p)

# name -> (restype, argtypes); every g4_status function raises G4Error through check().
SIGNATURES = {
    "g4_ctx_create": (_S, [_I, _P, _PP]),
    "g4_ctx_destroy": (_S, [_P]),
    "g4_ctx_set_stream": (_S, [_P, _P]),
    "g4_ctx_set_pdl": (_S, [_P, _I]),
    "g4_selftest_wait_timeout": (_S, [_P, C.c_uint32]),
    "g4_stream_sync": (_S, [_P]),
    "g4_ctx_check_device": (_S, [_P, C.POINTER(C.c_uint32)]),
    "g4_last_error_string": (C.c_char_p, []),
    "g4_version": (C.c_char_p, []),
    "g4_kernel_launch_count": (C.c_uint64, []),
    "g4_linear_create": (_S, [_P, _P, _P, _I, _I, _I, _I, _PP]),
    "g4_linear_destroy": (_S, [_P]),
    "g4_linear_shape": (_S, [_P, C.POINTER(_I), C.POINTER(_I)]),
    "g4_linear_w4a16": (_S, [_P, _P, _P, _I, _P, _I]),
    "g4_linear_w4a16_impl": (_S, [_P, _P, _P, _I, _P, _I, _I]),
    "g4_linear_w4a16_f32": (_S, [_P, _P, _P, _I, _P]),
    "g4_attention_f32": (_S, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "g4_convert": (_S, [_P, _P, _I, _P, _I, C.c_longlong]),
    "g4_linear_dequant": (_S, [_P, _P, _I, _I, _P, _I]),
    "g4_ple_table_create": (_S, [_P, _P, _P, _I, _I, _I, _I, _PP]),
    "g4_ple_table_upload_rows": (_S, [_P, _P, _I, _I, _P, _P, _I]),
    "g4_ple_table_destroy": (_S, [_P]),
    "g4_ple_gather": (_S, [_P, _P, _P, _I, _I, _P, _I]),
    "g4_kv_create": (_S, [_P, _I, _I, _PP]),
    "g4_kv_destroy": (_S, [_P]),
    "g4_kv_create_ring": (_S, [_P, _I, _I, _I, _I, _PP]),
    "g4_kv_layout": (_S, [_P, C.POINTER(_I), C.POINTER(_I), C.POINTER(_I)]),
    "g4_kv_append": (_S, [_P, _P, _P, _P, _I, _I, _I]),
    "g4_kv_info": (_S, [_P, C.POINTER(_I), C.POINTER(_I), C.POINTER(_I)]),
    "g4_kv_reset": (_S, [_P]),
    "g4_kv_buffers": (_S, [_P, _PP, _PP]),
    "g4_attention": (_S, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "g4_attention_noalloc": (_S, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "g4_attention_rows": (_S, [_P, _P, _P, _I, _I, _I, _P, _I, _I, _I, _P]),
    "g4_rms": (_S, [_P, _P, _P, _I, _I, _F, _P, _I]),
    "g4_add_scale": (_S, [_P, _P, _P, C.c_longlong, _F, _P]),
    "g4_scale": (_S, [_P, _P, C.c_longlong, _F, _P]),
    "g4_gelu_mul_f32": (_S, [_P, _P, _P, C.c_longlong, _P]),
    "g4_gelu_ple_f32": (_S, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "g4_norm_rope": (_S, [_P, _P, _I, _I, _I, _I, _P, _I, _F, _F, _P]),
    "g4_softcap": (_S, [_P, _P, C.c_longlong, _F]),
    "g4_post_norm_add": (_S, [_P, _P, _P, _I, _P, _F, _P, _I, _I, _F, _P]),
    "g4_embed": (_S, [_P, _P, _I, _I, _P, _I, _F, _P, _P]),
    "g4_qkv_post": (_S, [_P, _P, _I, _I, _I, _I, _P, _P, _F, _I, _F, _P, _I, _P, _P, _P, _I]),
    "g4_gelu_mul": (_S, [_P, _P, _I, _I, _P]),
    "g4_gelu_ple": (_S, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "g4_linear_w4a16_planes": (_S, [_P, _P, _P, _I, _P]),
    "g4_linear_w4a16_geglu": (_S, [_P, _P, _P, _I, _P]),
    "g4_linear_w4a16_gelu_ple": (_S, [_P, _P, _P, _I, _P, _I, _I, _P]),
    "g4_dense_argmax": (_S, [_P, _P, _P, _I, _F, _P, _P]),
    "g4_post_norm_add_planes": (_S, [_P, _P, _P, _P, _F, _P, _I, _I, _F, _P]),
    "g4_qkv_post_planes": (_S, [_P, _P, _I, _I, _I, _P, _P, _F, _I, _F, _P, _I, _P, _P, _P, _I]),
    "g4_qkv_post_kv": (_S, [_P, _P, _I, _I, _P, _P, _F, _I, _F, _P, _I, _P, _P]),
    "g4_gelu_mul_planes": (_S, [_P, _P, _I, _I, _P]),
    "g4_gelu_ple_planes": (_S, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "g4_ple_mix": (_S, [_P, _P, _F, _P, _P, _I, _I, _I, _F, _P]),
    "g4_softcap_argmax": (_S, [_P, _P, _I, _I, _F, _P, _P]),
    "g4_advance_positions": (_S, [_P, _P, _I, _I, _I]),
    "g4_dense_create": (_S, [_P, _P, _I, _I, _I, _PP]),
    "g4_dense_destroy": (_S, [_P]),
    "g4_dense_weights": (_S, [_P, _PP]),
    "g4_dense_matmul": (_S, [_P, _P, _P, _I, _P]),
    "g4_decoder_create": (_S, [_P, _P, _P, _PP]),
    "g4_decoder_destroy": (_S, [_P]),
    "g4_decoder_step": (_S, [_P, _P, _P, _P, _P, _P]),
    "g4_decoder_reset": (_S, [_P]),
    "g4_decoder_set_timeline": (_S, [_P, _P, _I]),
}

_lib = None


def header_symbols() -> list[str]:
    """Every function name declared in include/g4w4.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:g4_status|const char\*|uint64_t)\s+(g4_\w+)\s*\(", text, re.M)))


def load() -> C.CDLL:
    """Loads libg4w4.so once (no GPU needed) and declares every signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is not built; run `python gemma4-js_b200/build.py`")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != G4_OK:
        msg = load().g4_last_error_string().decode(errors="replace")
        raise G4Error(status, msg or STATUS_NAMES.get(status, str(status)))


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
