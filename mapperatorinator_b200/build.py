"""Build the in-tree CUDA library ``_lib/libmtr_sampler.so`` for sm_100a.

The library is plain CUDA C++ behind a C ABI (``include/mtr_sampler.h``); it is
compiled with nvcc directly (no torch extension machinery) and loaded with
ctypes by :mod:`mapperatorinator_b200._native`.  The CUDA runtime is linked
statically, so the library only needs the NVIDIA driver at run time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libmtr_sampler.so"
SOURCES = [CSRC / "mtr_sampler.cu", CSRC / "mtr_stream.cu", CSRC / "mtr_stream_bf16.cu", CSRC / "mtr_stream_f16.cu",
           CSRC / "mtr_stream_f32.cu", CSRC / "mtr_lmhead.cu"]
HEADERS = [REPO_DIR / "include" / "mtr_sampler.h", CSRC / "mtr_common.cuh", CSRC / "mtr_stream.cuh"]
BUILD_DIR = PKG_DIR / "_build"

COMPILE_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
]
LINK_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static"]


def _nvcc() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(home) / "bin" / "nvcc"
    if path.exists():
        return str(path)
    raise RuntimeError("nvcc not found; set CUDA_HOME or put nvcc on PATH")


def _deps(src: Path) -> list:
    """Headers a translation unit includes (the stream kernel's also include mtr_stream.cuh)."""
    deps = [REPO_DIR / "include" / "mtr_sampler.h", CSRC / "mtr_common.cuh"]
    if src.name.startswith("mtr_stream"):
        deps.append(CSRC / "mtr_stream.cuh")
    return deps


def _obj(src: Path) -> Path:
    return BUILD_DIR / (src.stem + ".o")


def _obj_stale(src: Path) -> bool:
    obj = _obj(src)
    if not obj.exists():
        return True
    built = obj.stat().st_mtime
    return any(p.stat().st_mtime > built for p in [src, *_deps(src)])


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > built for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if it is missing or older than its sources (one
    nvcc process per translation unit, in parallel, then one link)."""
    if not force and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    nvcc = _nvcc()
    objs, procs = [], []
    for src in SOURCES:
        obj = _obj(src)
        objs_needed = force or _obj_stale(src)
        if not objs_needed:
            objs.append(obj)
            continue
        cmd = [nvcc, *COMPILE_FLAGS, "-I", str(REPO_DIR / "include"), "-c", "-o", str(obj), str(src)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), file=sys.stderr)
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
        objs.append(obj)
    failed = []
    for cmd, pr in procs:
        out, err = pr.communicate()
        if pr.returncode != 0:
            failed.append(f"{' '.join(cmd)}\n{out}\n{err}")
        elif verbose and err:
            print(err, file=sys.stderr)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *LINK_FLAGS, "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
