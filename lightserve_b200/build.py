"""Builds liblightserve_b200.so (the C-ABI extension) in-tree with nvcc.

Every .cu file under csrc/ is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and linked into one shared
library next to this file. The CUDA runtime is linked statically and the
driver API (for TMA descriptors) is reached through cudaGetDriverEntryPoint,
so the library loads on a machine without a GPU driver (symbols can be
inspected there; launches need a B200).

Usage:  python -m lightserve_b200.build [--force] [--verbose-ptxas]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
BUILD_DIR = PKG_DIR.parent / "_build"
LIB_PATH = PKG_DIR / "liblightserve_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(INCLUDE),
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the lightserve_b200 extension needs CUDA 12.8+")
    return cand


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _compile(src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [_nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    newest_header = max((p.stat().st_mtime for p in _headers()), default=0.0)
    todo = []
    for s in srcs:
        obj = BUILD_DIR / (s.stem + ".o")
        if force or verbose_ptxas or not obj.exists() or obj.stat().st_mtime < max(
            s.stat().st_mtime, newest_header
        ):
            todo.append(s)
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            for obj, log in ex.map(lambda s: _compile(s, verbose_ptxas), todo):
                if log.strip():
                    logs.append(f"--- {obj.name}\n{log}")
    objs = [BUILD_DIR / (s.stem + ".o") for s in srcs]
    if force or todo or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < max(
        o.stat().st_mtime for o in objs
    ):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp),
               *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    if verbose_ptxas and logs:
        print("\n".join(logs))
    return LIB_PATH


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose_ptxas=args.verbose_ptxas)
    print(path)


if __name__ == "__main__":
    sys.exit(main())
