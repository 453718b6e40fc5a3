"""Build the shared library (``libdfm.so``: FM head, patch encoder, LLM decode
attention, vocoder) in-tree
with nvcc for sm_100a.

    python -m nanovllm_dots_b200.build

The library statically links the CUDA runtime and resolves the driver's
``cuTensorMapEncodeTiled`` at run time, so it needs no link-time libcuda.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libdfm.so")
SOURCES = ["dfm_api.cu"]
DEPS = ["dfm_api.cu", "dpe_api.cu", "llm_api.cu", "common.cuh", "gemm.cuh", "attn_tc.cuh", "ew.cuh",
        "pe.cuh", "llm_attn.cuh", "llm_step.cuh", "voc_api.cu", "voc.cuh"]
HEADERS = [os.path.join(os.path.dirname(PKG), "include", h) for h in ("dfm.h", "dpe.h", "dllm.h", "dvoc.h")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def flags(verbose_ptxas: bool = False) -> list[str]:
    f = ["-O3", "-std=c++17", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a",
         "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr"]
    if verbose_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, d) for d in DEPS] + HEADERS
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    if not force and not stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *flags(verbose_ptxas), *[os.path.join(CSRC, s) for s in SOURCES], "-o", tmp]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
