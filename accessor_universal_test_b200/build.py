"""Build recipe for libautdot.so and the command-line tools (sm_100a only).

``python -m accessor_universal_test_b200.build`` compiles every CUDA source
under csrc/ with nvcc for ``arch=compute_100a,code=sm_100a`` into
``accessor_universal_test_b200/lib/libautdot.so`` (in-tree, so the library
travels with the source tree) and links the C++ CLIs in ``tools/`` against
it.  Objects are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
TOOLS = os.path.join(PKG, "tools")
LIB_DIR = os.path.join(PKG, "lib")
OBJ_DIR = os.path.join(PKG, "_build")
LIB = os.path.join(LIB_DIR, "libautdot.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    f"-I{INCLUDE}", f"-I{CSRC}",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libautdot")
    return path


def _headers() -> list[str]:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.hpp"))
    hs += glob.glob(os.path.join(INCLUDE, "**", "*.h*"), recursive=True)
    return hs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
    if _stale(obj, [src] + _headers()):
        cmd = [nvcc()] + NVCC_FLAGS + ["-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            sys.stderr.write(r.stderr)
    return obj


def build_library(verbose: bool = False) -> str:
    os.makedirs(LIB_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), sources))
    if _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def build_tools() -> list[str]:
    """Link the C++ command-line tools against libautdot.so."""
    out = []
    for src in sorted(glob.glob(os.path.join(TOOLS, "*.cpp"))):
        exe = os.path.join(LIB_DIR, os.path.splitext(os.path.basename(src))[0])
        if _stale(exe, [src, LIB] + _headers()):
            cmd = ["g++", "-O2", "-std=c++17", f"-I{INCLUDE}", "-I/usr/local/cuda/include",
                   src, "-o", exe, f"-L{LIB_DIR}", "-lautdot",
                   "-Wl,-rpath,$ORIGIN", "-L/usr/local/cuda/lib64", "-lcublas", "-lcudart",
                   "-lpthread"]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"g++ failed on {src}:\n{r.stdout}\n{r.stderr}")
        out.append(exe)
    return out


def build(verbose: bool = False) -> str:
    lib = build_library(verbose)
    build_tools()
    return lib


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
