"""Build the CUDA library in place: doantotnghiepmoe_b200/libmoe_b200.so.

nvcc -gencode arch=compute_100a,code=sm_100a, one object per .cu under
_build/ (rebuilt when the source or any header is newer), then one shared
library.  No torch headers or types are involved: the library exports only
the C ABI of include/moe_b200.h.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libmoe_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, extra: list[str] | None = None) -> str:
    sys.path.insert(0, CSRC)
    import gen_tables  # noqa: E402
    gen_tables.main(os.path.join(CSRC, "_gen"))
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
               glob.glob(os.path.join(CSRC, "_gen", "*")) +
               glob.glob(os.path.join(ROOT, "include", "*.h")))
    objs = []
    jobs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if _newer(obj, [src] + headers):
            cmd = [NVCC, *ARCH, *FLAGS, *(extra or []), "-c", src, "-o", obj]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for err in ex.map(run, jobs):
            if verbose and err.strip():
                print(err)
    if jobs or _newer(LIB, objs):
        run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"])
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
