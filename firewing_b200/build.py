"""Build libfwmoe (the C-ABI CUDA library) in-tree for sm_100a.

Produces firewing_b200/libfwmoe.so (loaded by the Python host package and
the tests) and firewing_b200/libfwmoe.a (for a Rust build.rs to link).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build")
SOURCES = ["fw_api.cu", "fw_decode.cu", "fw_experts.cu", "fw_layout.cu", "fw_noalloc.cu", "fw_prefill.cu", "fw_ep.cu", "fw_p2p.cu", "fw_hc.cu", "fw_checkpoint.cu", "fw_codec.cu"]
HEADERS = ["fw_common.cuh", "fw_kernels.h", "fw_json.h"]
SO = os.path.join(HERE, "libfwmoe.so")
LIB = os.path.join(HERE, "libfwmoe.a")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--fmad=false",
    "-Xcompiler", "-fPIC,-O3,-ffp-contract=off",
    "-I", os.path.join(ROOT, "include"), "-I", CSRC,
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    deps_common = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "fwmoe.h")]
    objs = []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or ptxas_info or _stale(obj, [path] + deps_common):
            cmd = [nvcc, *ARCH, *FLAGS, "-c", path, "-o", obj]
            if ptxas_info:
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(SO, objs):
        subprocess.run([nvcc, *ARCH, "-Wno-deprecated-gpu-targets", "-shared", "-o", SO, *objs, "-ldl"], check=True)
    if force or _stale(LIB, objs):
        subprocess.run([nvcc, *ARCH, "-Wno-deprecated-gpu-targets", "-lib", "-o", LIB, *objs], check=True)
    return SO


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
