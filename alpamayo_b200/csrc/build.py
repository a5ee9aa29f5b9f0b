"""Build the native libraries in-tree for sm_100a.

  alpamayo_b200/lib/libparo_b200.so  — the C ABI of include/paro_b200.h
                                       (nvcc, -gencode arch=compute_100a,code=sm_100a)
  alpamayo_b200/lib/libparo_torch.so — the TORCH_LIBRARY(paro_b200) shim

Usage: python alpamayo_b200/csrc/build.py [--force]   (run by path: importing the
package would load the libraries before they are rebuilt)
Objects go to alpamayo_b200/_build/.  Only sources newer than their outputs
are recompiled.  Works without a GPU (nvcc cross-compiles).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "lib")
OBJ = os.path.join(PKG, "_build")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

CU_SOURCES = ["capi.cu", "rotq.cu", "rotq_fused.cu", "rotq_rows.cu", "rotq_decode.cu", "rotq_tc.cu", "prepare.cu", "gemm_decode.cu", "gemm_rows.cu", "gemm_tc.cu", "elementwise.cu"]
HEADERS = ["paro_common.cuh", "tc_ptx.cuh", "umma.cuh", "stream_segs.cuh"]
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"] + GENCODE


def _newer(src_list, out):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.exists(s) and os.path.getmtime(s) > t for s in src_list)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build step failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build(force: bool = False, verbose: bool = False) -> dict:
    os.makedirs(LIB, exist_ok=True)
    os.makedirs(OBJ, exist_ok=True)
    hdrs = [os.path.join(HERE, h) for h in HEADERS] + [os.path.join(ROOT, "include", "paro_b200.h")]
    objs, jobs = [], []
    for src in CU_SOURCES:
        s = os.path.join(HERE, src)
        o = os.path.join(OBJ, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _newer([s] + hdrs, o):
            jobs.append([NVCC] + NVCC_FLAGS + ["-c", s, "-o", o])
    logs = []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            logs += list(ex.map(_run, jobs))
    core = os.path.join(LIB, "libparo_b200.so")
    if force or jobs or _newer(objs, core):
        logs.append(_run([NVCC, "-shared"] + GENCODE + ["-cudart", "static", "-o", core] + objs))

    shim = os.path.join(LIB, "libparo_torch.so")
    shim_src = os.path.join(HERE, "torch_ops.cpp")
    if force or _newer([shim_src, core] + hdrs, shim):
        import torch
        from torch.utils import cpp_extension as ce
        inc = ce.include_paths() + [os.path.join(CUDA_HOME, "include")]
        tlib = os.path.join(os.path.dirname(torch.__file__), "lib")
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        cmd = (["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
                "-DTORCH_API_INCLUDE_EXTENSION_H=0"]
               + [f"-I{p}" for p in inc]
               + [shim_src, "-o", shim, f"-L{tlib}", f"-L{LIB}", "-lparo_b200", "-lc10", "-lc10_cuda",
                  "-ltorch", "-ltorch_cpu", "-ltorch_cuda", f"-Wl,-rpath,{tlib}", "-Wl,-rpath,$ORIGIN"])
        logs.append(_run(cmd))
    if verbose:
        print("\n".join(l for l in logs if l.strip()))
    return {"core": core, "shim": shim}


if __name__ == "__main__":
    out = build(force="--force" in sys.argv, verbose=True)
    print(out)
