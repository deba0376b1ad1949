"""Build libmmp_cuda.so in-tree for sm_100a.

Every ``*.cu`` under this directory is compiled by nvcc (in parallel) with
``-gencode arch=compute_100a,code=sm_100a -lineinfo`` and linked, together
with the static CUDA runtime and NVRTC, into
``macmetalpy_b200/_lib/libmmp_cuda.so``.  Objects are rebuilt only when a
source or header is newer than the object.

Usage: ``python macmetalpy_b200/csrc/build.py [--force] [--verbose]`` (run as a
script: importing it through the package would need the library it builds).
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
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
OBJ_DIR = os.path.join(PKG, "_build")
LIB_DIR = os.path.join(PKG, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libmmp_cuda.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def cuda_home() -> str:
    for cand in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if cand and os.path.exists(os.path.join(cand, "bin", "nvcc")):
            return cand
    nvcc = shutil.which("nvcc")
    if nvcc:
        return os.path.dirname(os.path.dirname(nvcc))
    raise RuntimeError("nvcc not found: set CUDA_HOME")


def _headers() -> list[str]:
    hs = glob.glob(os.path.join(HERE, "*.cuh")) + glob.glob(os.path.join(HERE, "*.h"))
    hs.append(os.path.join(REPO, "include", "mmp_cuda.h"))
    return hs


def _newest(paths) -> float:
    return max((os.path.getmtime(p) for p in paths if os.path.exists(p)), default=0.0)


def _compile(src: str, obj: str, nvcc: str, verbose: bool) -> tuple[str, int, str]:
    cmd = [nvcc, *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC", "-Xptxas", "-v" if verbose else "-O3",
           "-I", os.path.join(REPO, "include"), "-c", src, "-o", obj]
    p = subprocess.run(cmd, capture_output=True, text=True)
    return src, p.returncode, (p.stdout + p.stderr)


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> str:
    home = cuda_home()
    nvcc = os.path.join(home, "bin", "nvcc")
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(HERE, "*.cu")))
    hdr_time = _newest(_headers())
    todo = []
    objs = []
    for s in srcs:
        o = os.path.join(OBJ_DIR, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_time):
            todo.append((s, o))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
            futs = [ex.submit(_compile, s, o, nvcc, verbose) for s, o in todo]
            for f in futs:
                src, rc, out = f.result()
                if verbose or rc:
                    sys.stderr.write(out)
                if rc:
                    raise RuntimeError(f"nvcc failed on {os.path.basename(src)}")
    if todo or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < _newest(objs):
        lib64 = os.path.join(home, "lib64")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-o", LIB_PATH + ".tmp", *objs,
               "-L" + lib64, "-lnvrtc", "-ldl", "-Xlinker", "-rpath=" + lib64, "-cudart", "static"]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode:
            sys.stderr.write(p.stdout + p.stderr)
            raise RuntimeError("link of libmmp_cuda.so failed")
        os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
