"""Build the tokengate_b200 C-ABI shared library in-tree with nvcc (sm_100a).

    python -m tokengate_b200.build

writes tokengate_b200/_lib/libtokengate_b200.so next to this file. The
library depends only on the CUDA runtime (linked statically by nvcc) and
reaches the driver's tensor-map encoder through cudaGetDriverEntryPoint, so
it needs no link against libcuda and no framework headers.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
LIB_NAME = "libtokengate_b200.so"
LIB_PATH = os.path.join(OUT_DIR, LIB_NAME)
SOURCES = ["tokengate_b200.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build tokengate_b200")
    return cand


def _inputs():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh"))]
    files.append(os.path.join(os.path.dirname(HERE), "include", "tokengate_b200.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False, extra_flags=()) -> str:
    """Compile the library if any source is newer than it; return its path."""
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall", "--expt-relaxed-constexpr",
           "-I", os.path.join(os.path.dirname(HERE), "include"),
           *extra_flags,
           *[os.path.join(CSRC, s) for s in SOURCES], "-o", tmp]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
