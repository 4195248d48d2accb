"""Compile the CUDA sources under ``csrc/`` into ``liblora_b200.so`` (sm_100a).

The library is built in-tree next to this file so that it travels with the
source tree; nothing is installed into site-packages.  ``build()`` recompiles
only the translation units whose sources (or shared headers) are newer than
their objects.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PKG_DIR / "_build"
LIB_PATH = PKG_DIR / "liblora_b200.so"

SOURCES = ("runtime.cu", "gemm_tc.cu", "shrink.cu", "expand.cu", "decode.cu", "sgmv.cu", "sgmv_block.cu", "sgmv_tc.cu", "sgmv_unit.cu", "sgmv_linear.cu", "skinny_tc.cu", "gemm_split.cu")
ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")
NVCC_FLAGS = ("-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden")


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the LoRA kernels need the CUDA toolkit to build")
    return cand


def _headers_mtime() -> float:
    paths = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _compile(nvcc: str, src: Path, obj: Path, verbose: bool) -> str:
    cmd = [nvcc, *NVCC_FLAGS, *ARCH_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return proc.stderr


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Build (or refresh) ``liblora_b200.so`` and return its path."""
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    todo = []
    objs = []
    for name in SOURCES:
        src = CSRC / name
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            todo.append((src, obj))
    logs = []
    if todo:
        with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, verbose) for s, o in todo]
            for f in futs:
                logs.append(f.result())
    newest = max(o.stat().st_mtime for o in objs)
    if force or todo or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < newest:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp),
               "-cudart", "static"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB_PATH)
    if verbose:
        for log in logs:
            print(log)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
