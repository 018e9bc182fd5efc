"""Build libkestrel_cuda.so (sm_100a) in-tree with nvcc.

Every .cu under csrc/ is compiled for `-gencode arch=compute_100a,code=sm_100a`
with --fmad=false (no implicit a*b+c contraction: the kernels call __fmaf_rn
where Kestrel's reference fuses, and plain multiplies and adds elsewhere), then
linked with NCCL (expert parallelism) into one shared library next to this
file. The library is plain C ABI (include/kestrel_cuda.h).
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libkestrel_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "--fmad=false", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr"]


def _nccl_dirs():
    """NCCL headers/library: the wheel next to torch, else the system copy."""
    for base in sys.path:
        inc = os.path.join(base, "nvidia", "nccl", "include")
        lib = os.path.join(base, "nvidia", "nccl", "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.isdir(lib):
            return inc, lib
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def _stale(sources, headers) -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(f) > t for f in sources + headers + [__file__])


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
                     glob.glob(os.path.join(ROOT, "include", "*.h")))
    if not force and not _stale(sources, headers):
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    nccl_inc, nccl_lib = _nccl_dirs()
    inc = ["-I", os.path.join(ROOT, "include"), "-I", CSRC, "-I", nccl_inc]
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, *extra, *inc, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        return obj, (r.stdout + r.stderr)

    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        results = list(ex.map(compile_one, sources))
    if verbose or ptxas_info:
        for obj, log in results:
            if log.strip():
                print(f"== {os.path.basename(obj)}\n{log}")
    objs = [o for o, _ in results]
    tmp = LIB + ".tmp"
    cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-L", nccl_lib, "-l:libnccl.so.2",
           "-Xlinker", f"-rpath,{nccl_lib}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv))
