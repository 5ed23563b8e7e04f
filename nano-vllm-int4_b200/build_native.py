"""Build libnv4.so, the sm_100a kernel library, in-tree.

    python nano-vllm-int4_b200/build_native.py [--force] [--ptxas-verbose]

nvcc cross-compiles for sm_100a without a GPU.  All kernel sources are
compiled as one translation unit (csrc/nv4_unity.cu) so the device-side error
word is a single symbol without relocatable device code.  The CUDA runtime is
linked statically and the driver's tensor-map encoder is resolved at run time,
so the library depends on nothing but the driver.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT_DIR = os.path.join(HERE, "nanovllm", "_lib")
OUT = os.path.join(OUT_DIR, "libnv4.so")
STAMP = OUT + ".srchash"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def source_hash() -> str:
    h = hashlib.sha256()
    for d in (CSRC, INCLUDE):
        for name in sorted(os.listdir(d)):
            if name.endswith((".cu", ".cuh", ".h")):
                with open(os.path.join(d, name), "rb") as f:
                    h.update(name.encode() + b"\0" + f.read())
    h.update(" ".join(ARCH).encode())
    return h.hexdigest()


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    digest = source_hash()
    if not force and os.path.exists(OUT) and os.path.exists(STAMP):
        with open(STAMP) as f:
            if f.read().strip() == digest:
                return OUT
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "--cudart", "static", "-I", INCLUDE,
           "-o", OUT + ".tmp", os.path.join(CSRC, "nv4_unity.cu")]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("nvcc failed building libnv4.so")
    if verbose_ptxas:
        sys.stderr.write(proc.stderr)
    os.replace(OUT + ".tmp", OUT)
    with open(STAMP, "w") as f:
        f.write(digest + "\n")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args()
    print(build(args.force, args.ptxas_verbose))
