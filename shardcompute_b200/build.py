"""Build recipe for libsc_b200.so (sm_100a), in-tree.

``python -m shardcompute_b200.build`` compiles every ``csrc/*.cu`` with nvcc
for ``sm_100a`` only and links them, with NCCL, into
``shardcompute_b200/libsc_b200.so``.  Object files go to
``shardcompute_b200/_build/``; a source is recompiled when it or a header is
newer than its object.  No GPU is needed (nvcc cross-compiles).
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libsc_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libsc_b200.so")


def nccl_dirs():
    """(include, lib) of the NCCL that torch loads, so one NCCL is in the process."""
    import importlib.util

    spec = importlib.util.find_spec("nvidia")
    roots = list(spec.submodule_search_locations) if spec and spec.submodule_search_locations else []
    for r in roots:
        inc, lib = os.path.join(r, "nccl", "include"), os.path.join(r, "nccl", "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")) and glob.glob(os.path.join(lib, "libnccl.so*")):
            return inc, lib
    raise RuntimeError("NCCL headers/library (nvidia-nccl wheel) not found")


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def build(verbose: bool = False, force: bool = False) -> str:
    nvcc = _nvcc()
    nccl_inc, nccl_lib = nccl_dirs()
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    hdr_time = _newest(headers)

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_time):
            return obj, ""
        cmd = [nvcc, *ARCH, *CFLAGS, "-I", INCLUDE, "-I", nccl_inc, "-Xptxas", "-v", "-c", src, "-o", obj]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
        return obj, res.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, sources))
    objs = [o for o, _ in results]
    if verbose:
        for (o, log), s in zip(results, sources):
            if log:
                print(f"== {os.path.basename(s)}\n{log}", file=sys.stderr)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        nccl_so = os.path.basename(sorted(glob.glob(os.path.join(nccl_lib, "libnccl.so*")))[0])
        cmd = [nvcc, *ARCH, "-shared", "-o", LIB, *objs, "-L", nccl_lib, "-Xlinker", f"-l:{nccl_so}",
               "-Xlinker", f"-rpath,{nccl_lib}"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
