"""In-tree build of the B200 SDPA forward (run from anywhere: ``python build.py [--force]``).

Products (git-ignored, but they travel to the GPU box with the repository snapshot):

* ``fused_attn/libfa_sm100.so`` -- the C-ABI library of include/fa_sm100.h: the sm_100a kernel
  (csrc/fa_fwd_sm100.cu) and the dispatch layer (csrc/dispatch.cu), compiled by nvcc with
  ``-gencode arch=compute_100a,code=sm_100a -lineinfo`` and the CUDA runtime linked statically,
  so the library loads with or without torch in the process.
* ``fused_attn/_C<EXT_SUFFIX>`` -- the PyTorch operator library (csrc/ext.cpp), host C++ only,
  linked against libfa_sm100.so through an ``$ORIGIN`` rpath.
* ``fused_attn/libfa_sm100_checks.so`` -- the same library built with ``-DFA_DEBUG_CHECKS``: device
  index/address checks that record a status bit (fa_last_device_error -> cudaErrorAssert) and skip
  the access instead of trapping; the tests run it against the release build.
* ``fused_attn/fa_bench`` -- the torch-free benchmark (csrc/fa_bench.cpp): links libfa_sm100.so
  through include/fa_sm100.h alone and self-checks against the CPU oracle before timing.

nvcc cross-compiles without a GPU, so this runs on the CPU build host too.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
OUT_DIR = PKG_ROOT / "fused_attn"
BUILD_DIR = PKG_ROOT / "_build"
INCLUDE = REPO_ROOT / "include"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [*ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-Wall", f"-I{INCLUDE}", f"-I{CSRC}"]

KERNEL_SOURCES = ["fa_fwd_sm100.cu", "dispatch.cu", "fa_combine.cu", "fa_noalloc.cu"]
KERNEL_HEADERS = ["sm100_ptx.cuh", "fa_launch.h", "fa_kernel_common.cuh", "fa_fwd_lookahead.cuh"]

LIB_NAME = "libfa_sm100.so"
EXT_NAME = "_C" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so")


def lib_path() -> Path:
    return OUT_DIR / LIB_NAME


def ext_path() -> Path:
    return OUT_DIR / EXT_NAME


def host_cxx() -> str:
    """The host C++ compiler for the torch extension and for nvcc's host passes.

    /usr/bin/g++ is preferred over $CXX: a wrapper compiler that redirects the crt/libgcc search
    path (as this image's /opt/gcc/bin/g++ does) yields a library whose C++ exceptions crash
    when a TORCH_CHECK unwinds through torch's dispatcher.  FA_HOST_CXX overrides both."""
    for cand in (os.environ.get("FA_HOST_CXX"), "/usr/bin/g++", os.environ.get("CXX"),
                 shutil.which("g++")):
        if cand and Path(cand).exists():
            return cand
    return "g++"


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def checks_lib_path() -> Path:
    return OUT_DIR / "libfa_sm100_checks.so"


def build_kernels(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False,
                  checks: bool = False) -> Path:
    """libfa_sm100.so, or with `checks` libfa_sm100_checks.so (-DFA_DEBUG_CHECKS)."""
    obj_dir = BUILD_DIR / ("checks" if checks else "")
    obj_dir.mkdir(parents=True, exist_ok=True)
    headers = [CSRC / h for h in KERNEL_HEADERS] + [INCLUDE / "fa_sm100.h"]
    defs = ["-DFA_DEBUG_CHECKS"] if checks else []
    jobs, objs = [], []
    for src in KERNEL_SOURCES:
        s = CSRC / src
        o = obj_dir / (s.stem + ".o")
        if force or _stale(o, [s, *headers]):
            extra = ["-Xptxas", "-v"] if ptxas_verbose else []
            jobs.append([NVCC, "-ccbin", host_cxx(), *NVCC_FLAGS, *defs, *extra, "-c", str(s), "-o",
                         str(o)])
        objs.append(o)
    procs = []
    for cmd in jobs:  # the translation units compile in parallel
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((cmd, subprocess.Popen(cmd)))
    for cmd, pr in procs:
        if pr.wait() != 0:
            raise subprocess.CalledProcessError(pr.returncode, cmd)
    lib = checks_lib_path() if checks else lib_path()
    if force or _stale(lib, objs):
        _run([NVCC, "-ccbin", host_cxx(), *ARCH_FLAGS, "-shared", "-Xlinker", f"-soname={lib.name}",
              "-o", str(lib), *map(str, objs)], verbose)
    return lib


def bench_path() -> Path:
    return OUT_DIR / "fa_bench"


def build_bench(force: bool = False, verbose: bool = False) -> Path:
    """The torch-free C++ harness: host code only, the C ABI library and the CUDA runtime."""
    src = CSRC / "fa_bench.cpp"
    out = bench_path()
    if force or _stale(out, [src, INCLUDE / "fa_sm100.h", lib_path()]):
        _run([NVCC, "-ccbin", host_cxx(), *ARCH_FLAGS, "-O2", "-std=c++17", f"-I{INCLUDE}", str(src), "-o",
              str(out), f"-L{OUT_DIR}", "-l:" + LIB_NAME, "-Xlinker", "-rpath,$ORIGIN", "-ldl"],
             verbose)
    return out


def build_ext(force: bool = False, verbose: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "ext.cpp"
    out = ext_path()
    deps = [src, INCLUDE / "fa_sm100.h", lib_path()]
    if not force and not _stale(out, deps):
        return out
    cxx = host_cxx()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [*cpp_extension.include_paths(), sysconfig.get_paths()["include"], str(CUDA_HOME / "include"),
            str(INCLUDE)]
    libdirs = cpp_extension.library_paths()
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-Wno-unused-parameter",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
           *(f"-I{i}" for i in incs), str(src), "-o", str(out),
           *(f"-L{d}" for d in libdirs), "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_cuda", f"-L{OUT_DIR}", "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN"]
    _run(cmd, verbose)
    return out


def build(force: bool = False, verbose: bool = False, ext: bool = True) -> None:
    build_kernels(force=force, verbose=verbose)
    build_kernels(force=force, verbose=verbose, checks=True)
    build_bench(force=force, verbose=verbose)
    if ext:
        build_ext(force=force, verbose=verbose)


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true", help="rebuild everything")
    ap.add_argument("--no-ext", action="store_true", help="only the C-ABI library")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    build_kernels(force=args.force or args.ptxas_verbose, verbose=args.verbose,
                  ptxas_verbose=args.ptxas_verbose)
    build_kernels(force=args.force, verbose=args.verbose, checks=True)
    build_bench(force=args.force, verbose=args.verbose)
    if not args.no_ext:
        build_ext(force=args.force, verbose=args.verbose)
    print(f"built {lib_path()}" + ("" if args.no_ext else f" and {ext_path()}"))
    return 0


if __name__ == "__main__":
    sys.exit(main())
