"""Build recipe of libflyguy_b200.so (sm_100a only), in-tree next to the package.

  python -m flyguy_b200.csrc.build [--ptxas-v]

nvcc compiles for the B200 architecture-specific target (-gencode arch=compute_100a,code=sm_100a); the CUDA runtime is
linked statically, so the library needs only the driver at run time and shares torch's primary context.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
REPO = PKG.parent
LIB = PKG / "libflyguy_b200.so"
TRAIN = PKG / "fg_train"                             # the trainer executable (a main() over fg_train_main)
SOURCES = [HERE / "fg_core.cu", HERE / "fg_noalloc.cu", HERE / "fg_hopop.cu", HERE / "fg_train.cu", HERE / "fg_fly.cu"]
DEPS = SOURCES + [HERE / "fg_kernels.cuh", HERE / "fg_tcgen05.cuh", HERE / "fg_outtc.cuh", REPO / "include" / "flyguy_b200.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise FileNotFoundError("nvcc not found (the CUDA toolkit is needed to build libflyguy_b200.so)")


def stale() -> bool:
    return (not LIB.exists() or not TRAIN.exists() or
            any(d.stat().st_mtime > LIB.stat().st_mtime for d in DEPS + [HERE / "fg_train_main.c"]))


def build(force: bool = False, ptxas_v: bool = False, out: Path = LIB, defines: tuple[str, ...] = ()) -> Path:
    if not force and out == LIB and not stale():
        return out
    tmp = out.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-I", str(REPO / "include"), *[f"-D{d}" for d in defines], "-o", str(tmp), *map(str, SOURCES)]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if ptxas_v:
        sys.stderr.write(r.stderr)
    os.replace(tmp, out)
    if out == LIB:
        build_trainer()
    return out


def build_trainer() -> Path:
    """fg_train: gcc on the three-line main, linked to the library next to it (rpath $ORIGIN)."""
    cc = shutil.which("gcc") or "cc"
    cmd = [cc, "-O2", "-I", str(REPO / "include"), "-o", str(TRAIN), str(HERE / "fg_train_main.c"), "-L", str(PKG),
           "-lflyguy_b200", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"building fg_train failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    return TRAIN


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ptxas-v", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force or a.ptxas_v, ptxas_v=a.ptxas_v))
