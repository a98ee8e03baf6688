"""Build the B200 ConvRot library (libconvrot_b200.so) with nvcc for sm_100a.

Counterpart of the reference's hipcc build (_int4/build.py:73-86): one nvcc
call on the package's CUDA sources, output next to this file. It is run by
``__graft_entry__.build()`` and, when the library is missing, once by the
loader.
"""
from __future__ import annotations

import os
import shutil
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
_CSRC = os.path.join(os.path.dirname(_HERE), "csrc")
SOURCES = ["convrot_b200.cu", "noalloc.cu"]
HEADERS = ["sm100_ptx.cuh", "gemm_pair.cuh", "gemm_a8t.cuh", "lora_down.cuh", "linear_api.cuh"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def lib_name() -> str:
    return "libconvrot_b200.so"


def lib_path() -> str:
    return os.path.join(_HERE, lib_name())


def src_paths() -> list[str]:
    return [os.path.join(_CSRC, s) for s in SOURCES]


def is_stale() -> bool:
    """True when the library is missing or older than any CUDA source."""
    out = lib_path()
    if not os.path.exists(out):
        return True
    newest = max(os.path.getmtime(p) for p in src_paths() + [os.path.join(_CSRC, h) for h in HEADERS])
    return newest > os.path.getmtime(out)


def find_nvcc() -> str | None:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = os.path.join(home, "bin", "nvcc")
    return p if os.path.exists(p) else None


def build(verbose: bool = False) -> str:
    nvcc = find_nvcc()
    if not nvcc:
        raise RuntimeError("nvcc not found; cannot build libconvrot_b200.so")
    out = lib_path()
    tmp = out + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "-o", tmp, *src_paths()]
    if verbose:
        print("building:", " ".join(cmd))
    cp = subprocess.run(cmd, capture_output=True, text=True)
    if cp.returncode != 0 or not os.path.exists(tmp):
        raise RuntimeError(f"nvcc build failed:\n{cp.stderr}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print("built:", build(verbose=True))
