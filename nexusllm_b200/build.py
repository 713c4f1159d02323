"""Builds libnexus_gpu.so in-tree with nvcc for sm_100a.

    python -m nexusllm_b200.build

The library is a single translation unit (csrc/nexus_gpu.cu includes the
kernel headers).  Output: nexusllm_b200/lib/libnexus_gpu.so.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc", "nexus_gpu.cu")
OUT = os.path.join(HERE, "lib", "libnexus_gpu.so")
DEPS = [os.path.join(HERE, "csrc", f) for f in os.listdir(os.path.join(HERE, "csrc")) if f.endswith((".cu", ".cuh"))] + [
    os.path.join(ROOT, "include", "nexus_gpu.h")]
DROPIN_SRC = os.path.join(HERE, "csrc", "dropin.cpp")
DROPIN_OUT = os.path.join(HERE, "lib", "libnexus_dropin.so")

NVCC_FLAGS = [
    "-O3", "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-shared",
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(p) <= t for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cmd = [nvcc(), *NVCC_FLAGS, "-o", OUT, SRC]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    return OUT


def build_dropin(reference_include: str, out: str = DROPIN_OUT) -> str:
    """The C++ drop-in (csrc/dropin.cpp): NexusLLM's QuantizationKernel GGUF
    methods and an INexusComputeBackend device, compiled against the
    reference's own headers (`reference_include` = <NexusLLM>/include) and
    linked to libnexus_gpu.so.  Needs those headers, so it is built where the
    reference tree is present; the built .so travels with the library."""
    lib = build()
    os.makedirs(os.path.dirname(out), exist_ok=True)
    cmd = [shutil.which("g++") or "g++", "-O2", "-std=c++20", "-fPIC", "-shared",
           f"-I{reference_include}", "-o", out, DROPIN_SRC, f"-L{os.path.dirname(lib)}", "-lnexus_gpu",
           "-Wl,-rpath,$ORIGIN"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"drop-in build failed:\n{res.stderr}")
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
