"""Build libmicroserve_b200.so for sm_100a with nvcc (no torch involved).

Usage: python -m microserve_b200.csrc.build [--force] [--jobs N]

Objects go to microserve_b200/_build/, the shared library next to the
package's Python files so ctypes finds it in-tree.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
ROOT = PKG.parent
BUILD = PKG / "_build"
LIB = PKG / "libmicroserve_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I",
    str(ROOT / "include"),
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def compile_one(src: Path, force: bool, verbose_ptxas: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if not force and not _stale(obj, src, headers()):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose_ptxas and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as pool:
        objs = list(pool.map(lambda s: compile_one(s, force, verbose_ptxas), srcs))
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static", "-ldl",
               "-lrt", "-lpthread"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args()
    print(build(args.force, args.jobs, args.ptxas_verbose))


if __name__ == "__main__":
    main()
