"""Builds libvoxb200.so in-tree with nvcc for sm_100a.

    python voxtral-rust_b200/build.py [--verbose]

Objects go to voxtral-rust_b200/_build/; the shared library lands next to
this file so that it travels with the source tree.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libvoxb200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-ffp-contract=off",
          "-I", CSRC, "-I", os.path.join(ROOT, "include")]
SOURCES = ["vox_gemv.cu", "vox_attention.cu", "vox_misc.cu", "vox_noalloc.cu", "vox_bgemm.cu",
           "vox_prefill.cu", "vox_encoder.cu",
           "vox_capi.cpp", "vox_tp.cpp", "vox_stream.cpp", "vox_weights.cpp",
           "vox_tokenizer.cpp"]
HEADERS = ["vox_kernels.h", "vox_device.cuh", "vox_tcgen05.cuh", "vox_host.h", "vox_internal.h", "vox_json.h",
           "vox_watchdog.h"]


def _newer(src: str, dst: str) -> bool:
    return not os.path.exists(dst) or os.path.getmtime(src) > os.path.getmtime(dst)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdr_mtime = max(os.path.getmtime(os.path.join(CSRC, h)) for h in HEADERS)
    hdr_mtime = max(hdr_mtime, os.path.getmtime(os.path.join(ROOT, "include", "vox_decoder.h")))
    objs = []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s + ".o")
        objs.append(obj)
        stale = force or _newer(src, obj) or (os.path.exists(obj) and os.path.getmtime(obj) < hdr_mtime)
        if not stale:
            continue
        cmd = [NVCC, *ARCH, *COMMON, "-c", src, "-o", obj]
        if verbose and s.endswith(".cu"):
            cmd += ["-Xptxas", "-v"]
        if s.endswith(".cpp"):
            cmd = [NVCC, *ARCH, *COMMON, "-x", "c++", "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode:
            raise RuntimeError(f"nvcc failed on {s}")
    if force or any(_newer(o, LIB) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force="--force" in sys.argv))
