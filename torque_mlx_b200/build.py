"""Build ``libtorque_b200.so`` (the C-ABI CUDA library) in-tree with nvcc.

    python -m torque_mlx_b200.build            # or build_library() from Python

The library is compiled for sm_100a only and placed next to this file so it
travels with the source tree; it is loaded by ``torque_mlx_b200._lib``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libtorque_b200.so"
SOURCES = ["tq_append.cu", "tq_decode.cu", "tq_decode_mma.cu", "tq_glue.cu", "tq_peer.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libtorque_b200.so")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list((PKG.parent / "include").glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile every source to an object in parallel, then link the shared library."""
    if not force and not _stale():
        return LIB
    from concurrent.futures import ThreadPoolExecutor

    nvcc = _nvcc()
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    common = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", str(PKG.parent / "include")]
    if verbose:
        common.append("-Xptxas=-v")

    def compile_one(src: str) -> Path:
        obj = objdir / (Path(src).stem + ".o")
        cmd = [nvcc, *common, "-c", str(CSRC / src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or res.returncode:
            sys.stderr.write(res.stdout + res.stderr)
        if res.returncode:
            raise RuntimeError(f"nvcc failed on {src}")
        return obj

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        objs = list(pool.map(compile_one, SOURCES))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc, *ARCH, "-shared", *[str(o) for o in objs], "-o", str(tmp)], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build_library(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
