"""Build the sm_100a shared library ``lorafusion_b200/_lib/liblorafusion_b200.so``.

    python -m lorafusion_b200.csrc.build [--force] [--verbose]

Every translation unit is compiled by nvcc for ``compute_100a``/``sm_100a`` only
(with ``-lineinfo``), in parallel, then linked into one position-independent
shared library with a static CUDA runtime.  Objects are rebuilt when a source
or header is newer than the object.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
OBJ_DIR = os.path.join(PKG, "_build")
LIB_DIR = os.path.join(PKG, "_lib")
LIB_NAME = "liblorafusion_b200.so"
SOURCES = ["lf_tables.cpp", "lf_sched.cpp", "lf_simt.cu", "lf_tc.cu", "lf_rows.cu", "lf_capi.cu", "lf_noalloc.cu"]
HEADERS = ["lf_ptx.cuh", "lf_internal.cuh", os.path.join("..", "..", "include", "lorafusion_b200.h")]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "-I" + os.path.join(REPO, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA 12.9 toolkit is required to build lorafusion_b200")


def lib_path() -> str:
    return os.path.join(LIB_DIR, LIB_NAME)


def _newest_dep() -> float:
    return max(os.path.getmtime(os.path.join(HERE, h)) for h in HEADERS)


def _compile(src: str, force: bool, verbose: bool, extra: list[str]) -> str:
    obj = os.path.join(OBJ_DIR, src + ".o")
    path = os.path.join(HERE, src)
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(path), _newest_dep()):
        return obj
    cmd = [nvcc(), *ARCH, *COMMON, *extra, "-c", path, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [nvcc(), *COMMON, "-Wno-deprecated-gpu-targets", "-x", "c++", "-c", path, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr.strip():
        print(res.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose or ptxas_info, extra), SOURCES))
    out = lib_path()
    if force or not os.path.exists(out) or os.path.getmtime(out) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", out, *objs, "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills/smem per kernel")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas_info))


if __name__ == "__main__":
    sys.exit(main())
