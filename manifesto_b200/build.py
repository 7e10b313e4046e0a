"""Build libmfcuda.so (the sm_100a kernels + C ABI) in-tree with nvcc.

Usage: python -m manifesto_b200.build [-v] [--force]

The library is written next to this file (manifesto_b200/libmfcuda.so) so it
travels with the source tree; object files go to manifesto_b200/_build/.
Flags: sm_100a only, -O3 -lineinfo, IEEE float semantics (no fast-math,
-fmad=false: every fused multiply-add in the kernels is spelled out with
__fmaf_rn so the unfused arithmetic of the reference stays unfused).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
LIB_PATH = PKG_DIR / "libmfcuda.so"
INCLUDE_DIR = PKG_DIR.parent / "include"

SOURCES = [
    "runtime.cu",
    "convert.cu",
    "int4.cu",
    "axpy.cu",
    "quant.cu",
    "ckpt.cu",
    "fused.cu",
    "comm.cu",
    "probe.cu",
]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-fmad=false",
    "-Xcompiler", "-fPIC",
    "-Xptxas", "-warn-spills",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libmfcuda.so")
    return cand


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE_DIR.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    headers = _headers()
    objects = []
    for src in SOURCES:
        path = CSRC / src
        obj = BUILD_DIR / (Path(src).stem + ".o")
        objects.append(obj)
        if not force and not _stale(obj, [path] + headers):
            continue
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE_DIR), "-c", str(path), "-o", str(obj)]
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or _stale(LIB_PATH, objects):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects),
               "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers / spills per kernel")
    args = ap.parse_args(argv)
    path = build(verbose=args.verbose, force=args.force, ptxas_verbose=args.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
