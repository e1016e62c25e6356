"""Builds the in-tree C-ABI library ``flashinfer_b200/_lib/libfmoe.so`` for sm_100a.

Usage: ``python -m flashinfer_b200.build`` (or ``__graft_entry__.build()``).
nvcc cross-compiles without a GPU. The CUDA runtime is linked statically, the
driver's tensor-map encoder is resolved at run time through
``cudaGetDriverEntryPoint``, so the library needs nothing beyond the driver.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIBDIR, "libfmoe.so")
SOURCES = ["fmoe_api.cu", "fmoe_kernels.cu", "fmoe_gemm.cu", "fmoe_gemv.cu", "fmoe_static.cu",
           "fmoe_quant.cu", "fmoe_ep.cu", "fmoe_peak.cu"]
HEADERS = ["fmoe_internal.h", "fmoe_ptx.cuh", "fmoe_gemm_common.cuh", "fmoe_route.cuh",
           os.path.join("..", "..", "include", "fmoe.h")]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, s) for s in SOURCES] + [os.path.join(CSRC, h) for h in HEADERS]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    objs, cmds = [], []
    for src in SOURCES:
        obj = os.path.join(LIBDIR, src.replace(".cu", ".o"))
        cmd = [nvcc(), *NVCC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.append("-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        cmds.append(cmd)
        objs.append(obj)
    # the translation units are independent: compile them side by side
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=min(len(cmds), os.cpu_count() or 1)) as pool:
        for r in list(pool.map(lambda c: subprocess.run(c, capture_output=not verbose), cmds)):
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed ({' '.join(r.args)}):\n"
                                   f"{(r.stderr or b'').decode(errors='replace')}")
    tmp = LIB + ".tmp"
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static",
           *objs, "-o", tmp]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
