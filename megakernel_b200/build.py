"""In-tree build of the native code (sm_100a only).

* ``libmkb200.so``: the decode kernel + C ABI, compiled by nvcc directly
  (``-gencode arch=compute_100a,code=sm_100a -lineinfo``), no torch headers.
* ``_build/megakernel_extension*.so``: the PyTorch extension exposing the
  reference's ``decode(...)`` call, linked against ``libmkb200.so``.

Both land inside the package directory so they travel with the repository;
nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libmkb200.so")
EXT_DIR = os.path.join(HERE, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
KERNEL_SOURCES = ["mkb_decode.cu", "mkb_host.cu", "mkb_noalloc.cu", "mkb_prefill.cu"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _stale(target: str, deps: list) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_lib(force: bool = False, verbose: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in KERNEL_SOURCES]
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    deps.append(os.path.join(INCLUDE, "mkb200.h"))
    if not force and not _stale(LIB, deps):
        return LIB
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xptxas", "-v", "-shared",
           "-Xcompiler", "-fPIC", "-Xlinker", "-soname=libmkb200.so", "-o", LIB, *srcs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed building libmkb200.so")
    return LIB


def build_extension(verbose: bool = False):
    """Build (or reuse) the torch extension; returns the loaded module."""
    import ctypes

    import torch  # noqa: F401
    from torch.utils.cpp_extension import load

    build_lib()
    # The extension links -lmkb200; make the already-built library resolvable.
    ctypes.CDLL(LIB, mode=ctypes.RTLD_GLOBAL)
    os.makedirs(EXT_DIR, exist_ok=True)
    prebuilt = os.path.join(EXT_DIR, "megakernel_extension.so")
    deps = [os.path.join(CSRC, "binding.cpp"), os.path.join(INCLUDE, "mkb200.h")]
    if not _stale(prebuilt, deps):
        import importlib.machinery
        import importlib.util
        loader = importlib.machinery.ExtensionFileLoader("megakernel_extension", prebuilt)
        spec = importlib.util.spec_from_file_location("megakernel_extension", prebuilt, loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        return mod
    return load(
        name="megakernel_extension",
        sources=[os.path.join(CSRC, "binding.cpp")],
        extra_include_paths=[INCLUDE],
        extra_cflags=["-O3", "-std=c++17"],
        extra_ldflags=[f"-L{HERE}", "-lmkb200"],
        build_directory=EXT_DIR,
        with_cuda=True,
        verbose=verbose,
    )


def build_all(verbose: bool = False):
    build_lib(verbose=verbose)
    return build_extension(verbose=verbose)


if __name__ == "__main__":
    build_lib(force="--force" in sys.argv, verbose=True)
    build_extension(verbose=True)
    print("built", LIB)
