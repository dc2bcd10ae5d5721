"""Build recipe of libquasar_cuda.so (sm_100a) - run by __graft_entry__.build().

Every .cu under csrc/ is compiled with nvcc for sm_100a only and linked into
quasar_b200/libquasar_cuda.so (static CUDA runtime, C ABI of
include/quasar_sampler.h). synth.cu is compiled with -fmad=false so the
synthetic inputs match the CPU recipe bit for bit; the sampler kernels keep
contraction on but spell every rounding-sensitive step with __f*_rn intrinsics.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libquasar_cuda.so")
DECODE = os.path.join(HERE, "batched_decode")  # the batched decode driver (batched_decode.c)
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I" + INCLUDE]
PER_FILE = {"synth.cu": ["-fmad=false"]}
LINK_LIBS: list[str] = ["-ldl"]  # NCCL is dlopen'ed at run time (nccl_shard.cu), not linked


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libquasar_cuda")
    return cand


def sources() -> list[str]:
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _newest_dep() -> float:
    t = 0.0
    for d in (CSRC, INCLUDE):
        for f in os.listdir(d):
            t = max(t, os.path.getmtime(os.path.join(d, f)))
    return t


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    deps = _newest_dep()
    objs = []
    for src in sources():
        obj = os.path.join(BUILD, src[:-3] + ".o")
        objs.append(obj)
        if not force and os.path.exists(obj) and os.path.getmtime(obj) >= deps:
            continue
        cmd = [nvcc(), *COMMON, *PER_FILE.get(src, []), "-c", os.path.join(CSRC, src), "-o", obj]
        if ptxas_v:
            cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    if force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", LIB, *objs, *LINK_LIBS]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    # the batched decode driver (host C over the library)
    drv_src = os.path.join(HERE, "batched_decode.c")
    if force or not os.path.exists(DECODE) or max(os.path.getmtime(drv_src), os.path.getmtime(LIB)) > \
            os.path.getmtime(DECODE):
        cmd = [nvcc(), "-O2", "-Wno-deprecated-gpu-targets", "-I" + INCLUDE, drv_src, "-o", DECODE, "-L" + HERE,
               "-lquasar_cuda",
               "-Xlinker", "-rpath=$ORIGIN"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_v="--ptxas-v" in sys.argv)
