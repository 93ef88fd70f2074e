"""Builds libb2pa.so in-tree with nvcc for sm_100a.

Usage: ``python -m b2pa.build [--force] [-j N]`` (with the package directory on
``sys.path``) or ``b2pa.build.build()``.  Objects go to ``<pkg>/build/``, the
library to ``<pkg>/lib/libb2pa.so``.  A unit is recompiled when its ``.cu`` or
any header under ``csrc/`` or ``include/`` is newer than its object.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent.parent          # efficient-inference-system_b200/
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PKG_DIR / "build"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libb2pa.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
          "-Xcompiler", "-fvisibility=hidden"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(obj: Path, src: Path, newest_header: float) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or newest_header > t


def _compile(src: Path, obj: Path, extra: list[str]) -> tuple[Path, str]:
    cmd = [_nvcc(), *ARCH_FLAGS, *CFLAGS, *extra, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stdout + proc.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compiles every csrc/*.cu for sm_100a and links lib/libb2pa.so."""
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    todo = []
    for src in srcs:
        obj = BUILD_DIR / (src.stem + ".o")
        if force or ptxas_info or _stale(obj, src, newest_header):
            todo.append((src, obj))
    jobs = jobs or min(len(todo) or 1, os.cpu_count() or 4)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            for obj, log in ex.map(lambda so: _compile(so[0], so[1], extra), todo):
                if verbose and log.strip():
                    print(f"[{obj.name}]\n{log}")
    objs = [BUILD_DIR / (s.stem + ".o") for s in srcs]
    if force or todo or not LIB_PATH.exists() or any(o.stat().st_mtime > LIB_PATH.stat().st_mtime for o in objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = ap.parse_args(argv)
    path = build(force=args.force, jobs=args.jobs, verbose=args.verbose or args.ptxas_info,
                 ptxas_info=args.ptxas_info)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
