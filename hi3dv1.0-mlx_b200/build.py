"""Build the sm_100a shared library ``hi3d_b200/_lib/libhi3d_b200.so`` in place.

Compiles every ``csrc/*.cu`` with nvcc (one object per file, in parallel) and links them into one shared library that exports
the C ABI declared in ``include/hi3d_b200.h``.  Objects are rebuilt only
when a source or header is newer than the object.

Usage: ``python build.py [--force] [--jobs N]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as futures
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = REPO / "include"
BUILD = HERE / "_build"
LIB = HERE / "hi3d_b200" / "_lib" / "libhi3d_b200.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _compile(src: Path, force: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    newest = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = True) -> Path:
    """Compile and link the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    jobs = jobs or min(len(sources), os.cpu_count() or 4)
    with futures.ThreadPoolExecutor(jobs) as pool:
        objs = list(pool.map(lambda s: _compile(s, force), sources))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", *[str(o) for o in objs], "-ldl", "-o", str(LIB)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stderr}")
        if verbose:
            print(f"built {LIB.relative_to(REPO)}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args()
    try:
        build(args.force, args.jobs)
    except RuntimeError as exc:
        print(exc, file=sys.stderr)
        sys.exit(1)
