"""The Node-API addon (gemma4-js_b200/napi) compiles and binds what the JS runtime needs.

No `node` exists in this image, so the addon is compile-checked against a declarations-only
stand-in of node_api.h (tests/napi_stub/), linked against libg4w4.so and libcudart, and its
undefined g4_* symbols are matched with the library's exports and the header.  gpu_ops.js
must define every GPUOps method of the reference (custom-webgpu/gpu-runtime.js:1295-1378).
"""
import re
import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
NAPI = REPO / "gemma4-js_b200" / "napi"
CUDA_INC = Path("/usr/local/cuda/include")
CUDA_LIB = Path("/usr/local/cuda/lib64")

GPUOPS_METHODS = ["w4", "rms", "addScale", "scale", "geluMul", "geluPle", "normRope", "attention", "pleMix",
                  "headChunk", "track", "emptyF32", "dispose"]


@pytest.fixture(scope="module")
def addon(tmp_path_factory):
    if not shutil.which("gcc") or not (CUDA_INC / "cuda_runtime_api.h").exists():
        pytest.skip("gcc or the CUDA headers are missing")
    out = tmp_path_factory.mktemp("napi")
    obj, so = out / "g4w4_napi.o", out / "g4w4.node"
    cc = subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-fPIC", "-c", str(NAPI / "g4w4_napi.c"),
                         "-I", str(REPO / "tests" / "napi_stub"), "-I", str(REPO / "include"), "-I", str(CUDA_INC),
                         "-o", str(obj)], capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    ld = subprocess.run(["gcc", "-shared", "-o", str(so), str(obj), "-L", str(REPO / "gemma4-js_b200"), "-lg4w4",
                         "-L", str(CUDA_LIB), "-lcudart"], capture_output=True, text=True)
    assert ld.returncode == 0, ld.stderr
    return so


def _symbols(path, flag):
    out = subprocess.run(["nm", "-D", flag, str(path)], capture_output=True, text=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_addon_binds_library_symbols_that_exist(addon):
    import importlib
    L = importlib.import_module("gemma4-js_b200._lib")
    used = {s for s in _symbols(addon, "--undefined-only") if s.startswith("g4_")}
    exported = _symbols(L.LIB_PATH, "--defined-only")
    declared = set(L.header_symbols())
    assert len(used) >= 30
    assert used <= exported and used <= declared
    # the operator entry points of GPUOps, GPUW4Linear.load, pleRowsToGpu and KVCache
    for name in ("g4_linear_w4a16_f32", "g4_attention_f32", "g4_rms", "g4_add_scale", "g4_scale", "g4_gelu_mul_f32",
                 "g4_gelu_ple_f32", "g4_norm_rope", "g4_ple_mix", "g4_dense_matmul", "g4_softcap", "g4_linear_create",
                 "g4_ple_gather", "g4_ple_table_upload_rows", "g4_kv_append", "g4_convert"):
        assert name in used, name
    assert "napi_register_module_v1" in _symbols(addon, "--defined-only")


def test_js_runtime_has_every_gpuops_method():
    src = (NAPI / "gpu_ops.js").read_text()
    body = src[src.index("export class CudaGPUOps"):src.index("export class CudaW4Linear")]
    for m in GPUOPS_METHODS:
        assert re.search(rf"^\s+{m}\(", body, re.M), m
    # every addon function the JS calls is exported by the addon's property table
    c = (NAPI / "g4w4_napi.c").read_text()
    table = set(re.findall(r'FN\("(\w+)"', c))
    called = set(re.findall(r"\bg4\.(\w+)\(", src))
    assert called <= table, called - table
