"""Build the sm_100a shared library behind fa2.kernel.attention.

    python triton-fa2-forward_b200/build.py          # or: __graft_entry__.build()

Compiles csrc/*.cu with nvcc for sm_100a only (-gencode arch=compute_100a,code=sm_100a)
into fa2/libfa2_sm100.so (in-tree, so it travels with the source tree). The CUDA runtime
is linked statically; the library has no torch dependency and exports only the C ABI
declared in include/fa2_sm100.h.
"""

import os
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
LIB_PATH = os.path.join(PKG_DIR, "fa2", "libfa2_sm100.so")
SOURCES = [os.path.join(CSRC, "fa2_fwd_sm100.cu")]
DEPENDS = SOURCES + [
    os.path.join(CSRC, "ptx_sm100.cuh"),
    os.path.join(CSRC, "exp2_poly.cuh"),
    os.path.join(CSRC, "fa2_pair_sm100.cuh"),
    os.path.join(INCLUDE, "fa2_sm100.h"),
]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-cudart", "static",
]


def nvcc_path():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def up_to_date(out=LIB_PATH, deps=DEPENDS):
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(d) <= t for d in deps)


def build(force=False, verbose=False, extra_flags=()):
    """Compile the library if any source is newer than it. Returns the library path."""
    if not force and up_to_date():
        return LIB_PATH
    cmd = [nvcc_path(), *NVCC_FLAGS, *extra_flags, "-I", INCLUDE, "-I", CSRC, "-o", LIB_PATH, *SOURCES]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout, res.stderr, sep="\n")
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
