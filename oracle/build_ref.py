"""TEST INFRASTRUCTURE ONLY: build the reference's own CUDA kernels as checkers.

Compiles the unmodified reference sources where they lie
(``<reference>/packages/morphottention/csrc/cuda/attention/attention.cu`` and the headers
it includes) together with ``oracle/ref_shim.cpp`` into one shared library per
compile-time variant, written to ``oracle/_ref/``.  The reference fixes ``cube_m``,
``head_dim`` and causal masking at compile time (``csrc/cuda/utils/declarations.cuh:39-77``),
so each variant is a separate build with the reference's own ``-D`` switches.  The
reference's CMake build is not used.  Only tests and the golden-fixture generator load
these libraries.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
# Where the reference checkout lies: the MORPHO_REFERENCE_ROOT environment variable, else the
# build machine's checkout.  The one place this path is named; every other user reads REF_ROOT.
REF_ROOT = os.environ.get("MORPHO_REFERENCE_ROOT", "/root/reference")
CSRC = os.path.join(REF_ROOT, "packages", "morphottention", "csrc")
PY_PKG = os.path.join(REF_ROOT, "packages", "morphottention", "torch-ext", "morphottention")


def sources_present() -> bool:
    return os.path.isdir(CSRC)
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

# name -> (cube_m, head_dim, causal, extra defines)
VARIANTS = {
    "m16_hd32": (16, 32, False, ["-DKERNEL_BR_BWD=32", "-DKERNEL_BC_BWD=32"]),   # README shape (fwd + bwd)
    "m16_hd64": (16, 64, False, []),
    "m16_hd64_causal": (16, 64, True, []),
    "m32_hd64": (32, 64, False, []),
}


def lib_path(name: str) -> str:
    return os.path.join(OUT, f"ref_{name}.so")


def _build_one(name, verbose):
    import torch.utils.cpp_extension as ce
    m, hd, causal, extra = VARIANTS[name]
    target = lib_path(name)
    srcs = [os.path.join(CSRC, "cuda", "attention", "attention.cu"), os.path.join(HERE, "ref_shim.cpp")]
    if os.path.exists(target) and all(os.path.getmtime(target) >= os.path.getmtime(s) for s in srcs):
        return target
    incs = ce.include_paths()
    libs = ce.library_paths()
    import torch
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DKERNEL_CUBE_M={m}", f"-DKERNEL_HEAD_DIM_V={hd}",
           f"-DMORPHO_CAUSAL={1 if causal else 0}", "--expt-relaxed-constexpr", "-I" + CSRC] + extra
    cmd += ["-I" + p for p in incs] + srcs + ["-o", target]
    for p in libs:
        cmd += ["-L" + p, "-Xlinker", "-rpath=" + p]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"reference build {name} failed:\n{r.stderr[-4000:]}")
    return target


def build_reference(verbose: bool = False, names=None) -> list:
    """Build every variant (incremental).  Returns the library paths."""
    if not os.path.isdir(CSRC):
        raise FileNotFoundError(f"reference sources not found at {CSRC}")
    os.makedirs(OUT, exist_ok=True)
    names = list(names or VARIANTS)
    with cf.ThreadPoolExecutor(max_workers=min(4, len(names))) as ex:
        return list(ex.map(lambda n: _build_one(n, verbose), names))


if __name__ == "__main__":
    for p in build_reference(verbose="-v" in sys.argv):
        print(p)
