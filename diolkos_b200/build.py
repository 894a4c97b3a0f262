"""Build libdiolkos.so in-tree: the sm_100a CUDA kernels, the C ABI and the reference-API host
library, plus the CLI binaries.  Run as ``python -m diolkos_b200.build`` (or through
``__graft_entry__.build()``).  Incremental: an object is rebuilt only when a source or header is
newer than it.
"""
from __future__ import annotations

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
LIB = os.path.join(PKG, "libdiolkos.so")
BIN = os.path.join(PKG, "bin")

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
CUDA_HOME = os.path.dirname(os.path.dirname(os.path.realpath(NVCC)))
# The environment may point CC at a wrapper without OpenMP; the host library uses the system gcc.
HOST_CC = os.environ.get("DIOLKOS_CC", "gcc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-O2",
    "-ccbin", "g++",
] + os.environ.get("DIOLKOS_NVCC_EXTRA", "").split()  # e.g. -DDK_STEP_CHECKS for a self-checking build
CC_FLAGS = ["-O2", "-fPIC", "-std=c11", "-D_GNU_SOURCE", "-ffp-contract=off", "-Wall", "-Wno-unused-function",
            f"-I{INCLUDE}", f"-I{CUDA_HOME}/include"]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd: list[str]) -> None:
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(verbose: bool = True) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(CSRC, "host", "*.h")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    objs = []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        if _newer(obj, [src] + headers):
            _run([NVCC, *NVCC_FLAGS, "-c", src, "-o", obj])
        objs.append(obj)
    for src in sorted(glob.glob(os.path.join(CSRC, "host", "*.c"))):
        obj = os.path.join(BUILD, "host_" + os.path.basename(src) + ".o")
        if _newer(obj, [src] + headers):
            _run([HOST_CC, *CC_FLAGS, "-c", src, "-o", obj])
        objs.append(obj)
    if _newer(LIB, objs):
        # -Bsymbolic: calls between the library's own functions (forward -> dk_model_forward, sample ->
        # random_f32, ...) bind inside the library even where another loaded library exports the
        # reference's function names.
        _run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-Xlinker", "-Bsymbolic", "-o", LIB, *objs,
              "-lcudart_static", "-lrt", "-lpthread", "-ldl", "-lm"])
    # CLI binaries (reference bin/localinfer, bin/client, bin/benchmark counterparts)
    os.makedirs(BIN, exist_ok=True)
    for src in sorted(glob.glob(os.path.join(CSRC, "bin", "*.c"))):
        exe = os.path.join(BIN, os.path.splitext(os.path.basename(src))[0])
        if _newer(exe, [src, LIB] + headers):
            _run([HOST_CC, *CC_FLAGS, src, "-o", exe, f"-L{PKG}", "-ldiolkos", f"-Wl,-rpath,{PKG}",
                  "-Wl,-rpath,$ORIGIN/..", "-lm"])
    return LIB


SAN_FLAGS = ["-fsanitize=address,undefined", "-fno-sanitize-recover=undefined", "-fno-omit-frame-pointer", "-g",
             "-O1"]
SAN_LIB = os.path.join(BUILD, "libdiolkos_san.so")


def build_sanitized() -> str:
    """The same library with the host C code (the reference API: loader, JSON reader, tokenizer, sampler,
    tensor helpers) built under AddressSanitizer and UndefinedBehaviorSanitizer, the CUDA objects
    unchanged: _build/libdiolkos_san.so, for the CPU tests of the host code.  A process that loads it
    preloads the gcc sanitizer runtimes (sanitizer_runtimes())."""
    build(verbose=False)
    headers = glob.glob(os.path.join(CSRC, "host", "*.h")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    objs = [os.path.join(BUILD, os.path.basename(src) + ".o") for src in sorted(glob.glob(os.path.join(CSRC, "*.cu")))]
    for src in sorted(glob.glob(os.path.join(CSRC, "host", "*.c"))):
        obj = os.path.join(BUILD, "san_" + os.path.basename(src) + ".o")
        if _newer(obj, [src] + headers):
            _run([HOST_CC, *CC_FLAGS, *SAN_FLAGS, "-c", src, "-o", obj])
        objs.append(obj)
    if _newer(SAN_LIB, objs):
        _run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-Xlinker", "-Bsymbolic", "-o", SAN_LIB,
              *objs, "-lasan", "-lubsan", "-lcudart_static", "-lrt", "-lpthread", "-ldl", "-lm"])
    return SAN_LIB


def sanitizer_runtimes() -> list:
    """The gcc ASan and UBSan runtimes to preload (ASan first), or [] when this gcc has none."""
    out = []
    for name in ("libasan.so", "libubsan.so"):
        path = subprocess.run([HOST_CC, f"-print-file-name={name}"], capture_output=True, text=True).stdout.strip()
        if not os.path.isabs(path) or not os.path.exists(path):
            return []
        out.append(path)
    return out


if __name__ == "__main__":
    build()
    sys.exit(0)
