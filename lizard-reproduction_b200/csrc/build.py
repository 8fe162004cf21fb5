"""Build liblizard_cuda.so (sm_100a) in-tree with nvcc.

Each .cu file in this directory is compiled to an object under _build/ in
parallel, then linked into ../lizard_cuda/liblizard_cuda.so with the CUDA
runtime linked statically, so the library carries no dependency beyond the
driver. Usage: python build.py [--verbose] [--force]
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent / "lizard_cuda"
OUT = PKG / "liblizard_cuda.so"
BUILD = HERE / "_build"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
         "--expt-relaxed-constexpr", "-DNDEBUG"]


def nvcc():
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build")
    return cand


def sources():
    return sorted(p for p in HERE.glob("*.cu"))


def headers():
    return sorted(list(HERE.glob("*.cuh")) + list(HERE.glob("*.h"))
                  + list((HERE.parent.parent / "include").glob("*.h")))


def stale(obj, src, deps):
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def compile_one(src, verbose):
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}")
    return obj, res.stderr


def build(verbose=False, force=False):
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    deps = headers()
    todo = [s for s in srcs if force or verbose or stale(BUILD / (s.stem + ".o"), s, deps)]
    logs = {}
    if todo:
        workers = min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(workers) as ex:
            for obj, log in ex.map(lambda s: compile_one(s, verbose), todo):
                logs[obj.name] = log
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or todo or not OUT.exists() or any(o.stat().st_mtime > OUT.stat().st_mtime
                                                for o in objs):
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp),
               *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
        os.replace(tmp, OUT)
    if verbose:
        for name, log in logs.items():
            print(f"== {name}\n{log}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))
    sys.exit(0)
