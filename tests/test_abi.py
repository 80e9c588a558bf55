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


def test_struct_layouts_match_the_header(tmp_path):
    """The ctypes mirrors of g4_rows and g4_planes have the C header's size and field
    offsets (compiled by the host C compiler from include/g4w4.h)."""
    from pathlib import Path
    L = importlib_lib()
    inc = Path(L.HEADER).parent
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stddef.h>\n#include <stdio.h>\n#include "g4w4.h"\n'
        "int main(void) {\n"
        '  printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(g4_rows), offsetof(g4_rows, seq_base),\n'
        "         offsetof(g4_rows, rows_per_seq), offsetof(g4_rows, pos0), offsetof(g4_rows, flags), 0ul);\n"
        '  printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(g4_planes), offsetof(g4_planes, base),\n'
        "         offsetof(g4_planes, count), offsetof(g4_planes, stride), offsetof(g4_planes, ld), 0ul);\n"
        '  printf("%d\\n", G4_ROWS_HISTORY_READY);\n'
        '  printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(g4_decoder_layer), offsetof(g4_decoder_layer, kn),\n'
        "         offsetof(g4_decoder_layer, skip), offsetof(g4_decoder_layer, kv), offsetof(g4_decoder_layer, has_kv),\n"
        "         offsetof(g4_decoder_layer, rope_angles), offsetof(g4_decoder_layer, rope_base),\n"
        "         offsetof(g4_decoder_layer, inter), 0ul);\n"
        '  printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(g4_decoder_desc), offsetof(g4_decoder_desc, eps),\n'
        "         offsetof(g4_decoder_desc, softcap), offsetof(g4_decoder_desc, top), offsetof(g4_decoder_desc, embed),\n"
        "         offsetof(g4_decoder_desc, ple));\n"
        "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", str(inc), str(src), "-o", str(exe)], check=True)
    lines = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    rows = [int(v) for v in lines[0].split()]
    planes = [int(v) for v in lines[1].split()]
    R, P = L.G4Rows, L.G4Planes
    assert rows[:5] == [C.sizeof(R), R.seq_base.offset, R.rows_per_seq.offset, R.pos0.offset, R.flags.offset]
    assert planes[:5] == [C.sizeof(P), P.base.offset, P.count.offset, P.stride.offset, P.ld.offset]
    assert int(lines[2]) == L.G4_ROWS_HISTORY_READY
    dl, dd = [int(v) for v in lines[3].split()], [int(v) for v in lines[4].split()]
    DL, DD = L.G4DecoderLayer, L.G4DecoderDesc
    assert dl[:8] == [C.sizeof(DL), DL.kn.offset, DL.skip.offset, DL.kv.offset, DL.has_kv.offset,
                      DL.rope_angles.offset, DL.rope_base.offset, DL.inter.offset]
    assert dd == [C.sizeof(DD), DD.eps.offset, DD.softcap.offset, DD.top.offset, DD.embed.offset, DD.ple.offset]
