"""Build the in-tree shared library ``kernelforge_b200/_lib/libkernelforge_b200.so``.

Every ``csrc/*.cu`` is compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``),
in parallel, and linked into one shared library that exports the C ABI of
``include/kernelforge_b200.h``. Objects are rebuilt when a source or header is newer.

    python -m kernelforge_b200.build [--force] [--jobs N]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
OBJ_DIR = OUT_DIR / "obj"
LIB = OUT_DIR / "libkernelforge_b200.so"
INCLUDE = PKG.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC)]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build kernelforge_b200")


def _headers():
    return list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    nvcc = nvcc_path()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    todo = []
    objects = []
    for src in sources:
        obj = OBJ_DIR / (src.stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *headers]):
            todo.append((src, obj))

    def compile_one(item):
        src, obj = item
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
        if verbose:
            print(f"compiled {src.name}")
        return obj

    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            list(ex.map(compile_one, todo))
    if force or todo or _stale(LIB, objects):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects), "-lcudart"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
        if verbose:
            print(f"linked {LIB}")
    return LIB


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=True))


if __name__ == "__main__":
    main()
