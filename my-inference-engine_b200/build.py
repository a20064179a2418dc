"""Build recipe for the in-tree sm_100a shared library ``libqmv_b200.so``.

Run ``python my-inference-engine_b200/build.py`` or call ``build_library()``.
nvcc cross-compiles for sm_100a without a GPU.  The CUDA runtime is linked
statically and its symbols are kept private (``--exclude-libs``), so the
library can be loaded next to torch's own runtime.
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_PATH = os.path.join(PKG_DIR, "libqmv_b200.so")

SOURCES = ["qmv_kernels.cu", "qmv_capi.cpp", "qmv_qwen2.cpp", "qmv_gguf.cpp", "quantized_matvec.cpp"]
HEADERS = ["qmv_internal.h"]
PUBLIC_HEADERS = ["qmv_b200.h", "quantized_matvec.h", "gguf_quantized_view.h"]

NVCC_FLAGS = [
    "-std=c++17",
    "-O3",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler", "-fPIC,-fvisibility=hidden,-Wall",
    "-Xptxas", "-v",
    "-shared",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def _inputs():
    files = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    files += [os.path.join(REPO_DIR, "include", h) for h in PUBLIC_HEADERS]
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build_library(force: bool = False, verbose: bool = False) -> str:
    """Compile libqmv_b200.so in place (skipped when up to date)."""
    if not force and up_to_date():
        return LIB_PATH
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", os.path.join(REPO_DIR, "include"), "-I", CSRC,
           "-o", LIB_PATH + ".tmp",
           *[os.path.join(CSRC, s) for s in SOURCES],
           "-Xlinker", "--exclude-libs,ALL"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + proc.stdout + proc.stderr)
    if verbose:
        sys.stderr.write(proc.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    with open(os.path.join(PKG_DIR, "ptxas_report.txt"), "w") as fh:
        fh.write(proc.stderr)
    return LIB_PATH


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose="-v" in sys.argv))
