"""Build the in-tree C-ABI shared library ``streamindex_b200/_lib/libstreamindex_b200.so``.

Every ``csrc/*.cu`` is compiled for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``) with nvcc, in parallel, and linked into one
shared object with the CUDA runtime linked statically, so the library needs
only the driver at run time.  Rebuilds only when a source or header is newer
than the library.

    python -m streamindex_b200.build [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT_DIR = os.path.join(PKG, "_lib")
LIB = os.path.join(OUT_DIR, "libstreamindex_b200.so")
# debug build of the same sources with the kernels' per-tile %globaltimer
# stamps compiled in (SI_ATTN_TRACE, SI_IDX_TRACE); never loaded by the package
TRACE_LIB = os.path.join(OUT_DIR, "libstreamindex_b200_trace.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-diag-suppress", "177"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the StreamIndex-B200 CUDA library cannot be built")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in _deps())


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> str:
    lib = TRACE_LIB if trace else LIB
    if not force and not trace and up_to_date():
        return LIB
    nvcc = _nvcc()
    obj_dir = os.path.join(OUT_DIR, "obj_trace" if trace else "obj")
    os.makedirs(obj_dir, exist_ok=True)

    def compile_one(src):
        obj = os.path.join(obj_dir, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc, *ARCH, *FLAGS, *(["-DSI_ATTN_TRACE", "-DSI_IDX_TRACE"] if trace else []), "-I", INCLUDE, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            sys.stderr.write(r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = lib + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--trace", action="store_true", help="build the per-tile trace debug library")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, trace=a.trace))
