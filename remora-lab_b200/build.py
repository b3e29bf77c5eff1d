"""Build libhar_cuda.so in-tree for sm_100a with nvcc.

The library is the product: every CUDA kernel plus the C ABI declared in
include/har_cuda.h.  Output: remora-lab_b200/har_cuda/libhar_cuda.so (the
Python host layer loads it from there; it travels with the source tree).
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "har_cuda", "libhar_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h")) + [__file__]
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_build():
        return OUT
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                    "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]
    if verbose:
        flags += ["-Xptxas", "-v"]
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        objs.append(obj)
        procs.append((src, subprocess.Popen([NVCC, *flags, "-c", src, "-o", obj],
                                            stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = False
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0 or verbose:
            sys.stdout.write(out.decode())
        if p.returncode != 0:
            failed = True
    if failed:
        raise RuntimeError("nvcc failed")
    tmp = OUT + ".tmp"
    subprocess.run([NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart_static", "-lnccl",
                    "-lrt", "-lpthread", "-ldl"], check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
