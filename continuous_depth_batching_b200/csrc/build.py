"""Build libcdb_b200.so (the C-ABI CUDA library) in-tree with nvcc for sm_100a.

    python -m continuous_depth_batching_b200.csrc.build

The library lands next to the package (``continuous_depth_batching_b200/libcdb_b200.so``) so
it ships with the source tree; it is loaded with ctypes by ``continuous_depth_batching_b200._lib``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
REPO = PKG.parent
LIB_NAME = "libcdb_b200.so"
SOURCES = ["attention.cu", "prefill_attention.cu", "elementwise.cu", "gemm.cu", "scheduler.cu", "fused_ops.cu", "kv_swap.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")
    return cand


def library_path() -> Path:
    return PKG / LIB_NAME


def _stale(out: Path, inputs: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(p.stat().st_mtime > t for p in inputs)


def build_library(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile every ``.cu`` into objects, then link the shared library. Returns its path."""

    nvcc = nvcc_path()
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list((REPO / "include").glob("*.h"))
    objs = []
    procs = []
    for src in SOURCES:
        src_path = CSRC / src
        obj = build_dir / (src_path.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src_path, *headers]):
            cmd = [
                nvcc,
                *ARCH_FLAGS,
                "-O3",
                "-lineinfo",
                "-std=c++17",
                "-Xcompiler",
                "-fPIC",
                "-Xptxas",
                "-v" if verbose else "-O3",
                f"-I{REPO / 'include'}",
                "-c",
                str(src_path),
                "-o",
                str(obj),
            ]
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for src, proc in procs:
        out, _ = proc.communicate()
        if verbose or proc.returncode != 0:
            sys.stdout.write(out)
        if proc.returncode != 0:
            failed.append(src)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    lib = library_path()
    if force or _stale(lib, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(lib), *map(str, objs)]
        subprocess.run(cmd, check=True)
    return lib


if __name__ == "__main__":
    path = build_library(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
