"""Builds libg4w4.so (sm_100a CUDA + C ABI) in-tree with nvcc.

Each csrc/*.cu compiles to an object under _build/ (in parallel, skipped when up to
date), then everything links into gemma4-js_b200/libg4w4.so next to this file.
`python gemma4-js_b200/build.py` or `build()` from Python.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
OBJ = REPO / "_build" / "g4w4"
LIB = PKG / "libg4w4.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-v"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + [REPO / "include" / "g4w4.h"]


def _compile(src: Path, verbose: bool) -> tuple[Path, str]:
    obj = OBJ / (src.stem + ".o")
    newest_dep = max(p.stat().st_mtime for p in _deps() + [src])
    if obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj, ""
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(REPO / "include"), "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, (r.stdout + r.stderr) if verbose else ""


def build(verbose: bool = False) -> Path:
    OBJ.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    objs = [o for o, _ in results]
    for _, log in results:
        if log:
            print(log, file=sys.stderr)
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB) + ".tmp", *map(str, objs), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
