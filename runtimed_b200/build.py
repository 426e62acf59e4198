"""Build libruntimed_b200.so in-tree with nvcc for sm_100a.

    python -m runtimed_b200.build            # incremental
    python -m runtimed_b200.build --force    # rebuild everything

Each source compiles to an object under runtimed_b200/_build/ (git-ignored);
the shared library lands next to this file so it travels with the tree.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libruntimed_b200.so")
INCLUDE = os.path.join(ROOT, "include")

SOURCES = ["rtd_api.cu", "rtd_gemv.cu", "rtd_gemm.cu", "rtd_gemm_ts.cu", "rtd_tp.cu", "rtd_model.cu", "rtd_dequant.cu", "rtd_repack.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def host_cxx() -> str:
    return "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"


def _deps() -> list[str]:
    out = []
    for d in (CSRC, INCLUDE):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh", ".hpp")):
                out.append(os.path.join(d, f))
    return out


def _stale(target: str, inputs: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(i) > t for i in inputs)


def compile_one(src: str, force: bool, verbose: bool) -> str:
    path = os.path.join(CSRC, src)
    obj = os.path.join(BUILD, src + ".o")
    if not force and not _stale(obj, [path] + _deps()):
        return obj
    cmd = [nvcc(), "-ccbin", host_cxx(), *ARCH, "-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", f"-I{CSRC}", f"-I{INCLUDE}", "-c", path, "-o", obj]
    if src.endswith(".cu"):
        cmd[1:1] = ["-Xptxas", "-v"] if verbose else []
    else:
        cmd += ["-x", "c++"]
    subprocess.run(cmd, check=True)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force, verbose), SOURCES))
    if force or _stale(LIB, objs):
        cmd = [nvcc(), "-ccbin", host_cxx(), *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static"]
        subprocess.run(cmd, check=True)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    args = ap.parse_args()
    print(build(args.force, args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
