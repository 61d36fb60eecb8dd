"""Build the sm_100a CUDA library libtau_dxb.so in-tree.

    python -m tau_dxb_b200.build          # or: python tau_dxb_b200/build.py

Each .cu under csrc/ is compiled with nvcc for sm_100a (in parallel), then
linked into tau_dxb_b200/_lib/libtau_dxb.so with the static CUDA runtime, so
the library needs only the NVIDIA driver at run time. Objects are rebuilt
when a source or header is newer than them.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_lib", "obj")
LIB = os.path.join(HERE, "_lib", "libtau_dxb.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps_mtime() -> float:
    hdrs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hdrs), default=0.0)


def _compile(src: str, verbose_ptxas: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), _deps_mtime()) \
            and not verbose_ptxas:
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose_ptxas: bool = False, jobs: int = 8) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-lrt", "-ldl", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose_ptxas="-v" in sys.argv))
