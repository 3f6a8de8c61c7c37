"""In-tree build of the sm_100a kernels.

Produces, next to this file:

* ``libmorpho_sm100.so`` -- the C-ABI library (``include/morpho_sm100.h``): all CUDA
  kernels, static CUDA runtime, no torch dependency.
* ``_C.so`` -- the torch op shim registering ``torch.ops.morphottention.*``; links
  ``libmorpho_sm100.so`` through an ``$ORIGIN`` rpath.

Run ``python morphottention_b200/build.py`` (or call :func:`build`).  Objects go to
``<repo>/_build``; a source is recompiled when it or any header is newer than its object.
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(REPO, "_build")
LIB = os.path.join(PKG, "libmorpho_sm100.so")
SHIM = os.path.join(PKG, "_C.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I" + INCLUDE]
CU_SOURCES = ["host_common.cu", "gemm.cu", "attn_fwd.cu", "attn_bwd.cu", "softmorph.cu", "softmorph_tc.cu", "softmorph_tc_bwd.cu", "pointwise.cu", "capi.cu", "noalloc.cu", "selftest.cu", "score_probe.cu", "peer.cu"]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, flush=True)
    return r


def _compile_cu(src, verbose, ptxas_verbose):
    obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
    if not _stale(obj, [src] + _headers()):
        return obj
    cmd = [NVCC] + ARCH + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else []) + ["-c", src, "-o", obj]
    _run(cmd, verbose or ptxas_verbose)
    return obj


def _torch_paths():
    import torch.utils.cpp_extension as ce  # noqa: WPS433 (build-time only)
    return ce.include_paths(), ce.library_paths()


def build(verbose: bool = False, ptxas_verbose: bool = False, jobs: int | None = None) -> None:
    """Compile the kernels for sm_100a and link both shared libraries (incremental)."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in CU_SOURCES]
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile_cu(s, verbose, ptxas_verbose), srcs))
    if _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs, verbose)
    shim_src = os.path.join(CSRC, "torch_ops.cpp")
    if _stale(SHIM, [shim_src, LIB] + _headers()):
        incs, libs = _torch_paths()
        import torch
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
               "-I" + INCLUDE, "-I" + os.path.join(CUDA_HOME, "include"),
               "-I" + sysconfig.get_paths()["include"]]
        cmd += ["-I" + p for p in incs]
        cmd += [shim_src, "-o", SHIM, "-L" + PKG, "-lmorpho_sm100", "-Wl,-rpath,$ORIGIN"]
        for p in libs:
            cmd += ["-L" + p, "-Wl,-rpath," + p]
        cmd += ["-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch"]
        _run(cmd, verbose)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv)
    print("built", LIB, SHIM)
