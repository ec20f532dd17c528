"""Build the sm_100a shared library ``_lib/libfk_decode.so`` in-tree with nvcc.

    python -m fasterkernels_b200.build [--force]

The library is a plain C-ABI shared object (include/fk_decode.h): no torch
headers, no Python.  It links the CUDA runtime statically and reaches the
driver's cuTensorMapEncodeTiled through cudaGetDriverEntryPoint, so it needs
no libcuda at link time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_DIR = os.path.join(PKG_DIR, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libfk_decode.so")
SOURCES = [os.path.join(CSRC, n) for n in ("fk_decode.cu", "fk_kernels_f16.cu", "fk_kernels_bf16.cu",
                                           "fk_kernels_e4m3.cu", "fk_paged_append.cu")]
DEPS = SOURCES + [os.path.join(CSRC, "fk_ptx.cuh"), os.path.join(CSRC, "fk_decode_kernel.cuh"),
                  os.path.join(REPO_DIR, "include", "fk_decode.h"), os.path.abspath(__file__)]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
    "-Xfatbin", "-compress-all",  # per-file fatbins are otherwise stored uncompressed
]


def find_nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(s) > t for s in DEPS)


def build_library(force: bool = False, verbose: bool = False) -> str:
    """Compile every source to an object in parallel (the kernel sets of the
    three KV types are separate translation units), then link the .so."""
    if not force and not needs_build():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    nvcc = find_nvcc()
    inc = ["-I", os.path.join(REPO_DIR, "include")]
    objs, procs = [], []
    for src in SOURCES:
        obj = os.path.join(LIB_DIR, os.path.splitext(os.path.basename(src))[0] + ".o")
        cmd = [nvcc, *NVCC_FLAGS, *inc, "-c", "-o", obj, src]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append(subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
        objs.append(obj)
    errors = []
    for p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            errors.append(out)
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc link failed:\n" + res.stdout + res.stderr)
    os.replace(tmp, LIB_PATH)
    for obj in objs:
        os.remove(obj)
    return LIB_PATH

if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose=True))
