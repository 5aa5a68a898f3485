"""Build the shadowkv_b200 CUDA library in-tree (sm_100a).

    python -m shadowkv_b200.build          # or: python shadowkv_b200/build.py

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` into
``shadowkv_b200/libshadowkv_b200.so``.  The library exports the C ABI of
``include/shadowkv_b200.h`` and links the CUDA runtime statically, so it
does not depend on which libcudart another module of the process loaded.
Object files are cached under ``shadowkv_b200/_build`` and rebuilt when a
source or header is newer.
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
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libshadowkv_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-rdc=true"]


def nvcc_path() -> str:
    for cand in [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]:
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the shadowkv_b200 library needs the CUDA toolkit to build")


def _newest_header() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(nvcc: str, src: str, extra: list[str], objdir: str = BUILD) -> str:
    obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, *extra, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
    stamp = obj + ".cmd"
    fresh = (os.path.exists(obj) and os.path.exists(stamp) and open(stamp).read() == " ".join(cmd)
             and os.path.getmtime(obj) >= max(os.path.getmtime(src), _newest_header()))
    if fresh:
        return obj
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    with open(stamp, "w") as f:
        f.write(" ".join(cmd))
    return obj


TRACE_LIB = os.path.join(PKG, "libshadowkv_b200_trace.so")


def build(verbose: bool = False, extra: list[str] | None = None, lib: str | None = None) -> str:
    """Compile the library if any source changed; return its path.

    ``extra``: more nvcc flags; ``lib``: output path (default the product
    library).  A library built to another path keeps its objects in a folder
    of its own, so that it and the product library are not rebuilt in turn.
    """
    extra = list(extra or [])
    out = lib or LIB
    objdir = BUILD if out == LIB else os.path.join(BUILD, os.path.basename(out)[:-3])
    os.makedirs(objdir, exist_ok=True)
    nvcc = nvcc_path()
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, extra, objdir), srcs))
    if not os.path.exists(out) or os.path.getmtime(out) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc, *ARCH, "-shared", "-rdc=true", "-cudart", "static", "-Xcompiler", "-fPIC", *objs, "-o", out]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print("built", out)
    return out


def build_trace(verbose: bool = False) -> str:
    """The trace build (``-DSKV_TRACE``: per-phase stamps and per-CTA records,
    read with ``skv_trace_*``) as ``libshadowkv_b200_trace.so``; load it with
    ``SKV_LIB`` set to its path."""
    return build(verbose, ["-DSKV_TRACE"], TRACE_LIB)


def ptxas_report() -> str:
    """Registers / spills / shared memory of every kernel (``-Xptxas -v``)."""
    nvcc = nvcc_path()
    out = []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-Xptxas", "-v", "-I", os.path.join(ROOT, "include"), "-c", src,
               "-o", os.devnull]
        r = subprocess.run(cmd, capture_output=True, text=True)
        out.append(f"== {os.path.basename(src)}\n{r.stderr}")
    return "\n".join(out)


if __name__ == "__main__":
    if "--ptxas" in sys.argv:
        print(ptxas_report())
    else:
        build(verbose=True)
