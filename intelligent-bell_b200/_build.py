"""Build ``libspeccache_b200.so`` in-tree with nvcc for sm_100a.

The library has no Python or torch dependency at build time: it is plain CUDA C++
behind the C ABI declared in ``include/speccache_b200.h``.  The built ``.so`` sits
next to this file, so it travels with the source tree.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
LIB_NAME = "libspeccache_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    built = os.path.getmtime(LIB_PATH)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    deps += glob.glob(os.path.join(INCLUDE, "*.h")) + [os.path.abspath(__file__)]
    return any(os.path.getmtime(d) > built for d in deps)


def build_library(force: bool = False, verbose: bool = False, ptxas_info: bool = False,
                  out_path: str | None = None, defines: dict | None = None) -> str:
    """Compile every CUDA/C++ source into the shared library; returns its path.

    ``out_path`` / ``defines`` build a variant elsewhere with tuning macros set
    (e.g. ``{"SC_DENSE_MIN_BLOCKS": 4}``); the default is the in-tree library.
    """
    target = out_path or LIB_PATH
    if out_path is None and not force and not _stale():
        return LIB_PATH
    cmd = [
        _nvcc(),
        "-O3",
        "-std=c++17",
        *ARCH_FLAGS,
        "-lineinfo",
        "-Xcompiler",
        "-fPIC,-O3,-fvisibility=hidden",
        "-shared",
        f"-I{INCLUDE}",
        *[f"-D{k}={v}" for k, v in (defines or {}).items()],
        "-o",
        target + ".tmp",
        *sources(),
    ]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr}")
    if verbose or ptxas_info:
        print(proc.stderr, file=sys.stderr)
    os.replace(target + ".tmp", target)
    return target


if __name__ == "__main__":
    build_library(force=True, verbose=True, ptxas_info="--ptxas" in sys.argv)
