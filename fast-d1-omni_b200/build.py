"""Builds libd1kernels for sm_100a (B200) in-tree.

Outputs, next to this file:
  libd1kernels.so  the shared library Python loads (kernels + C-ABI + host runner)
  libd1kernels.a   the static archive with the same symbols, the drop-in for the archive the reference's
                   build.rs:11-40 produces from cuda/kernels.cu + cuda/gemm.cu

nvcc cross-compiles without a GPU. Usage: python build.py [--force]
"""
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
OBJ = HERE / "_build"
SO = HERE / "libd1kernels.so"
ARCHIVE = HERE / "libd1kernels.a"

SOURCES = ["gemm.cu", "kernels.cu", "attn.cu", "audio.cu", "runner.cpp", "engine.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall", f"-I{INCLUDE}"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = OBJ / (s.stem + ".o")
        objs.append(o)
        if force or _stale(o, [s, *headers]):
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(s), "-o", str(o)]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(SO, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(SO), *map(str, objs), "-ldl"]
        subprocess.run(cmd, check=True)
    if force or _stale(ARCHIVE, objs):
        if ARCHIVE.exists():
            ARCHIVE.unlink()
        subprocess.run(["ar", "crs", str(ARCHIVE), *map(str, objs)], check=True)
    return SO


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(SO)
