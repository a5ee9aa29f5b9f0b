"""Compile the reference's own rotation kernel for sm_100a (test infrastructure).

The reference ships one CUDA source for the activation half of the W4A8
linear: kernels/paroquant_kernels/src/rotation.cu (+ rotation.cuh and
kernels/fused_quant/nvfp4_utils.cuh, included by relative path).  It is a
torch extension that registers ``torch.ops.rotation.rotate`` and
``rotate_and_quant`` (rotation.cu:576-584).  This script compiles that file
where it lies with nvcc directly -- it does not run the reference's
setup.py -- using the flags setup.py chooses on a B200 (setup.py:69-90):
``--use_fast_math``, ``-DENABLE_BF16``, the half / bf16 operator un-defines,
and ``-DDISABLE_FUSED_KERNELS`` because every B200 has compute capability
10.0 (setup.py:54-66), which compiles the NVFP4 ``rotate_and_quant`` out.

Output: ``oracle/_ref/librotation_ref.so`` (git-ignored; it travels to the
GPU box with the snapshot, the reference checkout does not).  Loaded only by
the parity tests and bench.py's reference-GPU leg through
``oracle/ref_gpu.py``; the product never loads it.

Usage: python oracle/build_ref.py [--force]   (needs the reference checkout;
a no-op with a message when it is absent)
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
OUT = os.path.join(OUT_DIR, "librotation_ref.so")
REF_ROOT = os.environ.get("PARO_REFERENCE_ROOT", "/root/reference")
SRC = os.path.join(REF_ROOT, "kernels", "paroquant_kernels", "src", "rotation.cu")
DEPS = [SRC, os.path.join(REF_ROOT, "kernels", "paroquant_kernels", "src", "rotation.cuh"),
        os.path.join(REF_ROOT, "kernels", "fused_quant", "nvfp4_utils.cuh")]
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")

# setup.py:69-83 (base flags) + :86-90 (B200: fused kernels disabled)
REF_NVCC_FLAGS = ["-O3", "-std=c++17", "-DENABLE_BF16",
                  "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
                  "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
                  "-U__CUDA_NO_BFLOAT162_OPERATORS__", "-U__CUDA_NO_BFLOAT162_CONVERSIONS__",
                  "--expt-relaxed-constexpr", "--expt-extended-lambda", "--use_fast_math", "-w",
                  "-DDISABLE_FUSED_KERNELS"]
# setup.py:8-39 on a B200 adds both 10.0 and 10.0a
GENCODE = ["-gencode", "arch=compute_100,code=sm_100", "-gencode", "arch=compute_100a,code=sm_100a"]


def available() -> bool:
    return all(os.path.exists(p) for p in DEPS)


def _newer(srcs, out):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs)


def build(force: bool = False, verbose: bool = False) -> str | None:
    """Compile the reference kernel into OUT; returns its path, or None
    when the reference checkout is not present (the prebuilt file, if any,
    is then left as it is)."""
    if not available():
        if verbose:
            print(f"reference sources not found under {REF_ROOT}: oracle/_ref not rebuilt")
        return OUT if os.path.exists(OUT) else None
    if not force and not _newer(DEPS + [os.path.abspath(__file__)], OUT):
        return OUT
    import torch
    from torch.utils import cpp_extension as ce
    os.makedirs(OUT_DIR, exist_ok=True)
    inc = ce.include_paths() + [sysconfig.get_paths()["include"], os.path.join(CUDA_HOME, "include")]
    tlib = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    obj = os.path.join(OUT_DIR, "rotation_ref.o")
    cc = ([os.path.join(CUDA_HOME, "bin", "nvcc")] + REF_NVCC_FLAGS + GENCODE
          + ["-Xcompiler", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
             "-DTORCH_API_INCLUDE_EXTENSION_H"]
          + [f"-I{p}" for p in inc] + ["-c", SRC, "-o", obj])
    link = ([os.path.join(CUDA_HOME, "bin", "nvcc"), "-shared"] + GENCODE
            + [obj, "-o", OUT, f"-L{tlib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
               "-ltorch_python", f"-Xlinker", f"-rpath={tlib}"])
    for cmd in (cc, link):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("reference kernel build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    os.remove(obj)
    if verbose:
        print(f"built {OUT}")
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
