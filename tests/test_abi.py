"""CPU tests of the C ABI boundary: the library loads and exports what include/g4w4.h declares."""
import ctypes as C
import subprocess

import pytest


def test_library_exports_every_header_symbol(g4):
    L = importlib_lib()
    lib = L.load()
    names = L.header_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(L.SIGNATURES), "ctypes table and header disagree"
    out = subprocess.run(["nm", "-D", "--defined-only", str(L.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(names) <= exported


def test_version_and_error_string(g4):
    lib = importlib_lib().load()
    assert lib.g4_version().startswith(b"g4w4")
    assert isinstance(lib.g4_last_error_string(), bytes)


def test_null_arguments_are_rejected_without_a_gpu(g4):
    L = importlib_lib()
    lib = L.load()
    assert lib.g4_ctx_create(0, None, None) == -1  # G4_ERR_INVALID before touching CUDA
    assert b"null out" in lib.g4_last_error_string()
    assert lib.g4_linear_shape(None, None, None) == -1
    assert lib.g4_kv_info(None, None, None, None) == -1
    assert lib.g4_ctx_destroy(None) == 0


def test_context_creation_fails_cleanly_without_gpu(g4):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = importlib_lib()
    h = C.c_void_p()
    st = L.load().g4_ctx_create(0, None, C.byref(h))
    assert st in (-1, -3)
    with pytest.raises(L.G4Error):
        L.check(st)


def importlib_lib():
    import importlib
    return importlib.import_module("gemma4-js_b200._lib")
