"""Build the reference CUDA kernel from its own sources (test infrastructure).

Compiles ``megakernel.cu`` (with ``config.cuh``) where it lies in the reference
checkout, plus ``oracle/ref_shim.cu``, into ``oracle/_ref/libref_megakernel.so``
for sm_100a. No reference source is copied; the output directory is git-ignored
but travels to the GPU box. The reference's own build (``model.py:14-20``,
torch.utils.cpp_extension with pytorch_binding.cu) is not used: the shim stands
in for the binding without PyTorch headers.

    python oracle/build_ref.py [/path/to/reference]

The reference checkout is taken from ``MKB_REFERENCE_DIR`` when set, else from
``DEFAULT_REF`` (where this build container mounts it).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
OUT = os.path.join(OUT_DIR, "libref_megakernel.so")
# the reference checkout: MKB_REFERENCE_DIR, else a "reference" directory beside this repository
DEFAULT_REF = os.environ.get("MKB_REFERENCE_DIR",
                             os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))


def build(ref_dir: str = DEFAULT_REF, force: bool = False) -> str | None:
    src = os.path.join(ref_dir, "megakernel.cu")
    if not os.path.exists(src):
        return None
    shim = os.path.join(HERE, "ref_shim.cu")
    if (not force and os.path.exists(OUT)
            and os.path.getmtime(OUT) >= max(os.path.getmtime(src), os.path.getmtime(shim))):
        return OUT
    os.makedirs(OUT_DIR, exist_ok=True)
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared", "-Xcompiler", "-fPIC",
           "-I", ref_dir, "-o", OUT, src, shim]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("building the reference kernel failed")
    return OUT


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REF, force=True))
