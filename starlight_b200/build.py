"""Builds libslc.so, the backend-cuda C-ABI library, for sm_100a only.

Usage: python -m starlight_b200.build [--force] [-j N]

Every .cu/.cpp under starlight_b200/csrc is compiled by nvcc with
-gencode arch=compute_100a,code=sm_100a into starlight_b200/_build/ and linked
into starlight_b200/libslc.so (in-tree, so the built library travels with the
repository snapshot). Objects are rebuilt when a source or header is newer.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libslc.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-I", CSRC,
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cpp")) + glob.glob(os.path.join(CSRC, "*.cu")) +
                  glob.glob(os.path.join(CSRC, "kernels", "*.cu")))
    headers = (glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True) +
               glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True) +
               glob.glob(os.path.join(ROOT, "include", "*.h")))
    return srcs, headers


def _obj(src):
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    return os.path.join(BUILD, rel + ".o")


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, headers, force):
    obj = _obj(src)
    if not force and not _stale(obj, [src] + headers):
        return obj, None
    cmd = [nvcc()] + NVCC_FLAGS + ["-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd[1:1] = ["-x", "cu"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f"{' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
    return obj, None


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs, headers = _sources()
    jobs = jobs or min(8, os.cpu_count() or 4)
    errors = []
    objs = []
    with cf.ThreadPoolExecutor(jobs) as ex:
        for obj, err in ex.map(lambda s: _compile(s, headers, force), srcs):
            objs.append(obj)
            if err:
                errors.append(err)
    if errors:
        raise RuntimeError("libslc build failed:\n" + "\n".join(errors))
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"libslc link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    a = ap.parse_args(argv)
    build(force=a.force, jobs=a.j, verbose=True)


if __name__ == "__main__":
    sys.exit(main())
