"""Builds libpjrt_b200.so in-tree: nvcc for the sm_100a kernels, g++ for the host compiler / runtime.

    python mccl-jax_b200/build.py [--force] [--jobs N]

Output: mccl-jax_b200/lib/libpjrt_b200.so, exporting GetPjrtApi (the PJRT drop-in boundary,
include/pjrt_b200.h) and the b200_* kernel entry points (include/b200_kernels.h) — nothing else.
The library links the CUDA runtime statically, NVRTC and NCCL dynamically (rpath into this image's
CUDA toolkit and the pip NCCL that torch also uses), and does not link libcuda: driver entry points
are resolved at run time, so the library loads on hosts without a GPU.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libpjrt_b200.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dirs():
    try:
        import nvidia.nccl as n  # the NCCL torch ships (2.28.x); same path on every box of this image
        base = list(n.__path__)[0]
        return os.path.join(base, "include"), os.path.join(base, "lib")
    except Exception:
        return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def sources():
    cu = sorted(glob.glob(os.path.join(CSRC, "kernels", "*.cu")))
    cc = sorted(glob.glob(os.path.join(CSRC, "**", "*.cc"), recursive=True))
    return cu, cc


def headers():
    return (glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True) +
            glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True) +
            glob.glob(os.path.join(ROOT, "include", "*.h")))


def obj_path(src):
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    return os.path.join(BUILD, rel + ".o")


def compile_one(src, force, hdr_mtime):
    out = obj_path(src)
    if not force and os.path.exists(out) and os.path.getmtime(out) >= max(os.path.getmtime(src), hdr_mtime):
        return out, ""
    nccl_inc, _ = nccl_dirs()
    if src.endswith(".cu"):
        cmd = ["nvcc", *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
               "-I" + os.path.join(CUDA, "include"), "-c", src, "-o", out]
    else:
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wno-unused-function",
               "-I" + os.path.join(CUDA, "include"), "-I" + nccl_inc, "-c", src, "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return out, r.stderr


def build(force=False, jobs=None, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    cu, cc = sources()
    hdr_mtime = max(os.path.getmtime(h) for h in headers())
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as ex:
        futs = [ex.submit(compile_one, s, force, hdr_mtime) for s in cu + cc]
        objs = []
        for f in futs:
            o, log = f.result()
            objs.append(o)
            if verbose and log.strip():
                print(log)
    if os.path.exists(LIB) and not force and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    _, nccl_lib = nccl_dirs()
    vers = os.path.join(BUILD, "exports.map")
    with open(vers, "w") as f:
        f.write("{ global: GetPjrtApi; b200_*; local: *; };\n")
    cmd = ["nvcc", *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs,
           "-L" + os.path.join(CUDA, "lib64"), "-lnvrtc", "-Xlinker", "-rpath=" + os.path.join(CUDA, "lib64"),
           "-L" + nccl_lib, "-l:libnccl.so.2", "-Xlinker", "-rpath=" + nccl_lib,
           "-Xlinker", "--version-script=" + vers, "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))


if __name__ == "__main__":
    sys.exit(main())
