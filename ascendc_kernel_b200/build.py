"""Builds the CUDA library (sm_100a) in-tree: ascendc_kernel_b200/lib/libdsa_b200.so.

Run ``python -m ascendc_kernel_b200.build`` (or call :func:`build`). Each
``csrc/*.cu`` is compiled by nvcc for ``sm_100a`` only and the objects are
linked into one shared library that exports the C ABI of
``include/dsa_b200.h``. Objects are rebuilt when a source or header is newer.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC_DIR = os.path.join(PKG_DIR, "csrc")
INCLUDE_DIR = os.path.join(REPO_DIR, "include")
BUILD_DIR = os.path.join(PKG_DIR, "_build")
LIB_DIR = os.path.join(PKG_DIR, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libdsa_b200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3",
    "-Xptxas",
    "-v",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand) and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")
    return cand


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC_DIR, "*.cuh")) + glob.glob(
        os.path.join(CSRC_DIR, "*.h")) + glob.glob(os.path.join(INCLUDE_DIR, "*.h"))


def _newest(paths: list[str]) -> float:
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def build(verbose: bool = False, force: bool = False) -> str:
    """Compiles every CUDA source for sm_100a and links the shared library.

    Returns the path of the library. Raises RuntimeError with the compiler's
    output when a step fails.
    """
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC_DIR, "*.cu")))
    hdr_time = _newest(_headers())
    objs = []
    ptxas_logs = []
    for src in sources:
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if (not force and os.path.exists(obj)
                and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_time)):
            continue
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", INCLUDE_DIR, "-I", CSRC_DIR, "-c", src,
               "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        ptxas_logs.append(r.stderr)
        if verbose:
            print(r.stderr, file=sys.stderr)
    if (force or not os.path.exists(LIB_PATH)
            or os.path.getmtime(LIB_PATH) < _newest(objs)):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", LIB_PATH, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
