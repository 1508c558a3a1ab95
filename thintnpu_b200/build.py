"""Build libttn.so (the C-ABI op-pass library) in-tree with nvcc for sm_100a.

Usage: python -m thintnpu_b200.build [--verbose]

Each csrc/*.cu compiles to an object under _build/ (in parallel), then the
objects link into thintnpu_b200/libttn.so.  The .so is git-ignored but
travels with the source tree, so a GPU host needs no compiler.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
BUILD = ROOT / "_build"
LIBRARY = PACKAGE / "libttn.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         f"-I{ROOT / 'include'}"]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _compile(source: Path, verbose: bool, ptxas_info: bool) -> Path:
    obj = BUILD / (source.stem + ".o")
    deps = [source, *CSRC.glob("*.cuh"), ROOT / "include" / "ttn.h"]
    if obj.exists() and all(obj.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(source), "-o", str(obj)]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), flush=True)
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode:
        raise RuntimeError(f"nvcc failed for {source.name}:\n{done.stdout}\n{done.stderr}")
    if ptxas_info or verbose:
        sys.stderr.write(done.stderr)
    return obj


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every csrc/*.cu and link libttn.so; returns the library path."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        objects = list(pool.map(lambda s: _compile(s, verbose, ptxas_info), sources))
    if LIBRARY.exists() and all(LIBRARY.stat().st_mtime >= o.stat().st_mtime for o in objects):
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objects), "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode:
        raise RuntimeError(f"link failed:\n{done.stdout}\n{done.stderr}")
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = parser.parse_args()
    print(build(args.verbose, args.ptxas_info))
