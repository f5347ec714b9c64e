"""Build recipe for libgdn_b200.so (nvcc, sm_100a), kept in-tree under lib/.

The library is a plain C-ABI shared object (include/gdn_b200.h); Python reaches
it through ctypes, other hosts through their own FFI.  nvcc cross-compiles for
sm_100a without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from typing import List, Optional

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_DIR = os.path.join(PKG_DIR, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libgdn_b200.so")
SELFTEST_LIB_PATH = os.path.join(LIB_DIR, "libgdn_b200_selftest.so")
INCLUDE = os.path.join(REPO_DIR, "include")

SOURCES = ["gdn_api.cu", "gdn_decode.cu", "gdn_prefill_recurrent.cu", "gdn_prefill_chunked.cu",
           "gdn_chunk_prep.cu", "gdn_prefill_tc.cu", "gdn_prefill_noalloc.cu", "gdn_output_gate.cu"]
# Known-answer checks of the tcgen05/TMA primitives, a separate test library.
SELFTEST_SOURCES = ["gdn_selftest.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: List[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra: Optional[List[str]] = None) -> str:
    """Compile the product library and the primitive self-test library (skips if up to date)."""
    _build_lib(LIB_PATH, SOURCES, force, verbose, extra)
    _build_lib(SELFTEST_LIB_PATH, SELFTEST_SOURCES, force, verbose, extra)
    return LIB_PATH


def _build_lib(lib_path: str, sources: List[str], force: bool, verbose: bool,
               extra: Optional[List[str]]) -> str:
    srcs = [os.path.join(CSRC, s) for s in sources]
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps.append(os.path.join(INCLUDE, "gdn_b200.h"))
    if not force and not _stale(lib_path, deps):
        return lib_path
    os.makedirs(LIB_DIR, exist_ok=True)
    obj_dir = os.path.join(LIB_DIR, "_obj")
    os.makedirs(obj_dir, exist_ok=True)
    nvcc = nvcc_path()
    common = ARCH_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                           "-Xcompiler", "-fvisibility=hidden", "-I", INCLUDE, "-I", CSRC,
                           "--expt-relaxed-constexpr"] + (extra or [])
    if verbose:
        common += ["-Xptxas", "-v"]
    objs = []
    for s in srcs:
        o = os.path.join(obj_dir, os.path.basename(s).replace(".cu", ".o"))
        cmd = [nvcc, "-c", s, "-o", o] + common
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0 or verbose:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(s)}")
        objs.append(o)
    tmp = lib_path + ".tmp"
    cmd = [nvcc, "-shared", "-o", tmp] + objs + ARCH_FLAGS + ["-Xcompiler", "-fPIC"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc link failed")
    os.replace(tmp, lib_path)
    return lib_path


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
