"""Builds libouroboros_b200.so (C++ allocator + sm_100a CUDA kernels + C ABI).

Usage:  python ouroboros-triton_b200/build.py [--force] [--verbose]

Every .cu file is compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a); .cpp files by nvcc's host
compiler. The shared library lands next to the Python loader
(src/kernels/libouroboros_b200.so) so the package finds it in-tree.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OBJ_DIR = PKG / "_build"
LIB = PKG / "src" / "kernels" / "libouroboros_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
CXXFLAGS = ["-std=c++17", "-O3", "-fPIC", "-Wall", f"-I{CUDA_HOME / 'include'}"]
CUFLAGS = ARCH + [
    "-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build the kernels")
    return cand


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.h*")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _compile(src: Path, verbose: bool) -> Path:
    obj = OBJ_DIR / (src.name + ".o")
    compiler = _nvcc() if src.suffix == ".cu" else (shutil.which("g++") or "g++")
    cmd = [compiler, "-c", str(src), "-o", str(obj), f"-I{INCLUDE}", f"-I{CSRC}"]
    cmd += CUFLAGS if src.suffix == ".cu" else CXXFLAGS
    if verbose:
        cmd += ["-Xptxas", "-v"] if src.suffix == ".cu" else []
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"compiling {src.name} failed:\n{proc.stdout}\n{proc.stderr}")
    if verbose and proc.stderr:
        print(proc.stderr, flush=True)
    return obj


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    stamp = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= stamp for p in _sources() + _headers() + [Path(__file__)])


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    OBJ_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    workers = min(len(srcs), os.cpu_count() or 4)
    with ThreadPoolExecutor(max_workers=workers) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), "-shared", *ARCH, "-o", str(tmp), *map(str, objs), "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"linking {LIB.name} failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    path = build(force=args.force, verbose=args.verbose)
    print(f"built {path}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
