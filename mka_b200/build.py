"""Builds libfastmka_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

Usage: python -m mka_b200.build [--force] [--verbose]

The library has no torch dependency: it links the CUDA runtime statically and
reaches the driver's cuTensorMapEncodeTiled through cudaGetDriverEntryPoint.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
LIB_NAME = "libfastmka_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

SOURCES = ["capi.cu", "gemm.cu", "route_scan.cu", "attn_prefill.cu", "attn_decode.cu", "peer.cu", "norm.cu", "l3_recall.cu"]
HEADERS = ["ptx.cuh", "fmka_internal.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--use_fast_math",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _inputs() -> list[Path]:
    return [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [INCLUDE / "fastmka_b200.h"]


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _inputs())


def build(force: bool = False, verbose: bool = False, jobs: int = 0) -> Path:
    """Compiles every CUDA source for sm_100a and links the shared library."""
    if not force and not needs_build():
        return LIB_PATH
    obj_dir = PKG_DIR / "_build"
    obj_dir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    procs = []
    objs = []
    for src in SOURCES:
        obj = obj_dir / (Path(src).stem + ".o")
        objs.append(obj)
        extra = os.environ.get("FMKA_NVCC_DEFINES", "").split()
        cmd = [nvcc, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode != 0:
            sys.stdout.write(out)
        if p.returncode != 0:
            failed.append(src)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    tmp = LIB_PATH.with_suffix(".so.tmp")
    link = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
            "-cudart", "static", *map(str, objs), "-o", str(tmp)]
    if verbose:
        print(" ".join(link), flush=True)
    subprocess.run(link, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
