"""Build ``libvates_b200.so`` in-tree with nvcc for sm_100a.

Usage: ``python -m vates_b200.build [--verbose]``. Objects go to
``vates_b200/_build/``; the shared library is written next to this file so it
travels with the source tree. Rebuilds only when a source is newer than the
library.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libvates_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

SOURCES = [
    "abi.cu",
    "moe_decode.cu",
    "moe_compat.cu",
    "route_reduce.cu",
    "kv_quant.cu",
    "kv_attn.cu",
    "moe_prefill.cu",
    "residency.cu",
    "kv_prefill_attn.cu",
    "dequant.cu",
    "ep.cu",
    "gdn.cu",
    "dense.cu",
    "qwen_next.cu",
    "gdn_fused.cu",
]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", "-I", INCLUDE]


def _deps():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)
             if f.endswith((".cu", ".cuh", ".h"))]
    files.append(os.path.join(INCLUDE, "vates_b200.h"))
    return files


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    cmd = [NVCC, *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        sys.stderr.write(res.stdout + res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = [s for s in SOURCES if os.path.exists(os.path.join(CSRC, s))]
    if not force and os.path.exists(LIB):
        lib_m = os.path.getmtime(LIB)
        if all(os.path.getmtime(f) <= lib_m for f in _deps()):
            return LIB
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    tmp = LIB + ".tmp"
    cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart", "-lcuda", "-ldl"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    v = "--verbose" in sys.argv
    print(build(force="--force" in sys.argv or v, verbose=v))
