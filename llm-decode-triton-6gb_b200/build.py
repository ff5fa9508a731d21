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
SOURCES = ["capi.cu", "nf4_gemm.cu", "nf4_gemm_tma.cu", "nf4_tc5.cu", "nf4_format.cu", "gqa_decode.cu", "decode_glue.cu", "tp_allreduce.cu", "lm_head.cu"]
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


def _compile(src: Path, obj: Path, verbose: bool) -> subprocess.CompletedProcess:
    cmd = [nvcc_path(), "-c", "-Xcompiler", "-fPIC", "-O3", "-std=c++17", *ARCH, "-lineinfo", f"-I{INCLUDE}",
           "-o", str(obj), str(src)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    return subprocess.run(cmd, capture_output=True, text=True)


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compiles every source to an object file in parallel (one nvcc per source), then links the
    shared library; objects live in a temporary directory next to the library."""
    if not force and not needs_build():
        return LIB_PATH
    import tempfile
    from concurrent.futures import ThreadPoolExecutor
    with tempfile.TemporaryDirectory(dir=LIB_PATH.parent) as tmp:
        objs = [Path(tmp) / (Path(s).stem + ".o") for s in SOURCES]
        with ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 1)) as ex:
            results = list(ex.map(lambda so: _compile(CSRC / so[0], so[1], verbose), zip(SOURCES, objs)))
        failed = False
        for res in results:
            if verbose or res.returncode != 0:
                sys.stdout.write(res.stdout)
                sys.stderr.write(res.stderr)
            failed |= res.returncode != 0
        if failed:
            raise RuntimeError("nvcc failed")
        cmd = [nvcc_path(), "-shared", *ARCH, "-cudart", "shared", "-o", str(LIB_PATH) + ".tmp", *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or res.returncode != 0:
            sys.stdout.write(res.stdout)
            sys.stderr.write(res.stderr)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc link failed with exit code {res.returncode}")
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force="--force" in sys.argv)
    print(LIB_PATH)
