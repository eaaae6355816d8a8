"""Build the in-tree native libraries of the complex_conv2d package.

    python build.py            # from this directory (or any cwd)

Produces, next to the Python sources in ``complex_conv2d/``:
  * ``libccv_b200.so`` - the CUDA kernels and the C ABI (include/ccv_b200.h),
    compiled by nvcc for sm_100a only (no torch dependency);
  * ``_C.so``          - the torch/pybind extension ``complex_conv2d._C``
    (csrc/bindings.cpp), linked against libccv_b200.so with an $ORIGIN rpath.

Both are cross-compiled here without a GPU; nothing is JIT-built at import
time.  Each CUDA translation unit compiles to an object under ``_build/`` in
parallel; objects and libraries are rebuilt only when a source is newer.
"""

from __future__ import annotations

import concurrent.futures
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
PKG = os.path.join(HERE, "complex_conv2d")
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
OBJ = os.path.join(HERE, "_build")

CU_SOURCES = ["ccv_api.cu", "ccv_fprop.cu", "ccv_fprop2.cu", "ccv_fprop2h.cu", "ccv_layout.cu",
              "ccv_noalloc.cu", "ccv_backward.cu"]
CU_HEADERS = ["ccv_internal.h", "ccv_ptx.cuh", "ccv_fprop_common.cuh", "ccv_epilogue.cuh",
              "ccv_layout_role.cuh"]
NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return os.path.join(cuda_home, "bin", "nvcc")


def _stale(out: str, deps) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)


def build_lib(verbose: bool = False, force: bool = False) -> str:
    out = os.path.join(PKG, "libccv_b200.so")
    headers = [os.path.join(CSRC, f) for f in CU_HEADERS] + [os.path.join(INCLUDE, "ccv_b200.h")]
    os.makedirs(OBJ, exist_ok=True)
    jobs = []
    objs = []
    for f in CU_SOURCES:
        src = os.path.join(CSRC, f)
        obj = os.path.join(OBJ, f.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            jobs.append([_nvcc(), "-O3", "-std=c++17", *NVCC_ARCH, "-lineinfo",
                         "-Xcompiler", "-fPIC", "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj])
    if jobs:
        with concurrent.futures.ThreadPoolExecutor(max_workers=len(jobs)) as pool:
            for fut in [pool.submit(_run, cmd, verbose) for cmd in jobs]:
                fut.result()
    if force or jobs or _stale(out, objs):
        _run([_nvcc(), *NVCC_ARCH, "-shared", *objs, "-o", out], verbose)
    return out


def build_ext(verbose: bool = False, force: bool = False) -> str:
    import torch
    import torch.utils.cpp_extension as ce

    lib = build_lib(verbose, force)
    out = os.path.join(PKG, "_C.so")
    src = os.path.join(CSRC, "bindings.cpp")
    if force or _stale(out, [src, lib, os.path.join(INCLUDE, "ccv_b200.h")]):
        incs = ce.include_paths("cuda") + [sysconfig.get_paths()["include"], INCLUDE]
        libdirs = ce.library_paths("cuda")
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", src,
               f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
               "-DTORCH_API_INCLUDE_EXTENSION_H", "-w"]
        for i in incs:
            cmd += ["-I", i]
        for d in libdirs:
            cmd += ["-L", d]
        cmd += ["-L", PKG, "-lccv_b200", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python",
                "-lc10_cuda", "-ltorch_cuda", "-Wl,-rpath,$ORIGIN", "-o", out]
        _run(cmd, verbose)
    return out


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    force = "--force" in argv
    verbose = "-v" in argv or "--verbose" in argv
    print(build_ext(verbose=verbose, force=force))


if __name__ == "__main__":
    main()
