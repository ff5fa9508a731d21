"""Build libb200decode.so (all CUDA kernels + the C ABI) in-tree for sm_100a.

    python llm-decode-triton-6gb_b200/build.py [--verbose]

The shared library lands next to the Python package (``b200kernels/libb200decode.so``) so it
travels with the source tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
LIB_PATH = PKG_ROOT / "b200kernels" / "libb200decode.so"
SOURCES = ["capi.cu", "nf4_gemm.cu", "nf4_gemm_tma.cu", "nf4_format.cu", "gqa_decode.cu", "decode_glue.cu", "tp_allreduce.cu", "lm_head.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libb200decode.so")
    return cand


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + [INCLUDE / "b200decode.h", Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps if p.exists())


def build(verbose: bool = False, force: bool = False) -> Path:
    if not force and not needs_build():
        return LIB_PATH
    cmd = [nvcc_path(), "-shared", "-Xcompiler", "-fPIC", "-O3", "-std=c++17", *ARCH, "-lineinfo",
           "-cudart", "shared", f"-I{INCLUDE}", "-o", str(LIB_PATH) + ".tmp",
           *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stdout.write(res.stdout)
        sys.stderr.write(res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed with exit code {res.returncode}")
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force="--force" in sys.argv)
    print(LIB_PATH)
