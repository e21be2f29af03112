"""Build ``libgdn_b200.so`` in-tree with nvcc for sm_100a.

The library is a plain shared object with a C ABI (``include/gdn.h``); it links
the CUDA runtime statically and needs no framework at load time.  Usage::

    python -m gated_deltanet_jax_b200._build [--force] [--verbose]
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD_DIR = os.path.join(REPO, "_build")
LIB_NAME = "libgdn_b200.so"
LIB_PATH = os.path.join(PKG, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
    "-I", INCLUDE, "-I", CSRC,
]


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    if os.path.exists(cand):
        return cand
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every ``csrc/*.cu`` and link ``libgdn_b200.so``; returns its path.

    Each file is compiled as a module of its own, without relocatable device
    code (no ``-rdc``, no device link).  chunk_bwd_static.cu relies on this:
    its 64 MiB ``__device__`` scratch array then lives in a module that CUDA's
    lazy loading brings onto a GPU only when the allocation-free backward is
    first called there, not whenever the library is loaded.
    """
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs, hdrs = _sources(), _headers()
    objs = [os.path.join(BUILD_DIR, os.path.basename(s)[:-3] + ".o") for s in srcs]
    extra = ["-Xptxas", "-v"] if verbose else []

    def compile_one(src_obj):
        src, obj = src_obj
        if not force and not _stale(obj, [src] + hdrs):
            return ""
        cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        logs = list(ex.map(compile_one, zip(srcs, objs)))
    if verbose:
        for log in logs:
            if log:
                sys.stderr.write(log)
    if force or _stale(LIB_PATH, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static",
               *objs, "-o", LIB_PATH]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
