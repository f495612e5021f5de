"""Build recipe for the native library: every CUDA source under csrc/ is compiled for sm_100a with
nvcc to its own object (in parallel, only the stale ones), and the objects are linked into one
shared object, ``actkv_open_b200/_native/libactkv_b200.so`` (in-tree, so that it ships with the
source tree).  The C ABI it exports is declared in include/actkv_b200.h.

    python -m actkv_open_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT_DIR = os.path.join(PKG, "_native")
LIB = os.path.join(OUT_DIR, "libactkv_b200.so")
OBJ_DIR = os.path.join(OUT_DIR, "obj")
HEADER = os.path.join(ROOT, "include", "actkv_b200.h")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "-cudart", "static"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the actkv_open_b200 kernels need the CUDA toolkit to build")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    """Files every object depends on besides its own source: the shared headers and this recipe."""
    return glob.glob(os.path.join(CSRC, "*.cuh")) + [HEADER, os.path.abspath(__file__)]


def _obj(src: str) -> str:
    return os.path.join(OBJ_DIR, os.path.splitext(os.path.basename(src))[0] + ".o")


def _newer(path: str, than: list[str]) -> bool:
    """True when ``path`` is missing or older than any of ``than``."""
    if not os.path.exists(path):
        return True
    t = os.path.getmtime(path)
    return any(os.path.getmtime(p) > t for p in than)


def _stale() -> bool:
    return _newer(LIB, sources() + _deps())


def _run(cmd: list[str]) -> str:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    return res.stdout + res.stderr


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; returns its path."""
    if not force and not _stale():
        return LIB
    os.makedirs(OBJ_DIR, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose else []
    deps = _deps()
    todo = [src for src in sources() if force or _newer(_obj(src), [src] + deps)]

    def compile_one(src: str) -> str:
        obj = _obj(src)
        out = _run([nvcc(), *ARCH, *FLAGS, *extra, "-c", "-o", obj + ".tmp", src])
        os.replace(obj + ".tmp", obj)
        return out

    workers = max(1, min(len(todo), os.cpu_count() or 1))
    with concurrent.futures.ThreadPoolExecutor(workers) as pool:
        logs = list(pool.map(compile_one, todo))
    tmp = LIB + ".tmp"
    logs.append(_run([nvcc(), *ARCH, *FLAGS, "-shared", "-o", tmp, *[_obj(src) for src in sources()]]))
    if verbose:
        sys.stderr.write("".join(logs))
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="also print ptxas register/smem usage")
    args = ap.parse_args()
    print(build(args.force, args.verbose))
