"""Builds libtroncons_b200.so in-tree (troncons_b200/_lib/), for sm_100a only.

Every CUDA source is compiled by nvcc with ``-gencode arch=compute_100a,code=sm_100a
-lineinfo -O3`` (no fast-math: E8M0 subnormal scales must stay exact); the host encoder with
``g++ -O3``. The library links the CUDA runtime statically, so it loads next to PyTorch's
own runtime without a version clash. Run ``python troncons_b200/construire.py`` (a standalone
script: importing the package loads the library this builds).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

ICI = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ICI, "csrc")
BUILD = os.path.join(ICI, "_build")
LIB = os.path.join(ICI, "_lib", "libtroncons_b200.so")
INCLUDE = os.path.join(os.path.dirname(ICI), "include")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}"]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", f"-I{INCLUDE}"]


def _sources():
    cu = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    cpp = sorted(f for f in os.listdir(CSRC) if f.endswith(".cpp"))
    return cu, cpp


def _deps():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, "troncons_b200.h")]


def a_jour() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in _deps())


def construire(force: bool = False, verbeux: bool = False, ptxas_v: bool = False) -> str:
    if not force and a_jour():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    cu, cpp = _sources()
    cmds = []
    objs = []
    for f in cu:
        o = os.path.join(BUILD, f + ".o")
        extra = ["-Xptxas", "-v"] if ptxas_v else []
        cmds.append([NVCC, *NVCC_FLAGS, *extra, "-c", os.path.join(CSRC, f), "-o", o])
        objs.append(o)
    for f in cpp:
        o = os.path.join(BUILD, f + ".o")
        cmds.append(["g++", *CXX_FLAGS, "-c", os.path.join(CSRC, f), "-o", o])
        objs.append(o)

    def run(c):
        r = subprocess.run(c, capture_output=True, text=True)
        return c, r

    with cf.ThreadPoolExecutor(max_workers=min(8, len(cmds))) as ex:
        for c, r in ex.map(run, cmds):
            if verbeux or ptxas_v:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                raise RuntimeError(f"build failed: {' '.join(c)}\n{r.stdout}\n{r.stderr}")
    tmp = LIB + ".tmp"
    r = subprocess.run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-lpthread", "-ldl"],
                       capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(construire(force="--force" in sys.argv, verbeux=True, ptxas_v="--ptxas" in sys.argv))
