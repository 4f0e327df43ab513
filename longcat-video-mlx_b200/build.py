"""Build the BSA engine's C-ABI shared library in-tree for sm_100a.

    python longcat-video-mlx_b200/build.py [--verbose]

Output: longcat-video-mlx_b200/longcat_video/_lib/libbsa_b200.so (git-ignored; travels with the
source tree).  nvcc cross-compiles, so this runs on a machine without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "longcat_video", "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libbsa_b200.so")
SOURCES = ["bsa_capi.cu", "bsa_attn.cu", "bsa_score.cu", "bsa_route.cu", "bsa_noalloc.cu", "bsa_xfer.cu"]
HEADERS = ["bsa_ptx.cuh", "bsa_kernels.h", "bsa_select.cuh"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(REPO, "include", "bsa_b200.h"),
                                                                  os.path.abspath(__file__)]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    cmd = [nvcc_path(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
           "-shared", "-Xcompiler", "-fPIC", "-I", os.path.join(REPO, "include"),
           "-o", LIB_PATH + ".tmp"] + [os.path.join(CSRC, f) for f in SOURCES]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose="--verbose" in sys.argv))
