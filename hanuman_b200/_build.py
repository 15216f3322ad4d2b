"""In-tree build of the native extension for sm_100a.

``build()`` compiles every source under ``csrc/`` with
``-gencode arch=compute_100a,code=sm_100a`` into
``hanuman_b200/_ext_build/hanuman_b200_C.so`` (ninja, incremental).  The
loader in :mod:`hanuman_b200.ops._ext` imports that file directly, so a GPU
machine that received the built tree never recompiles.
"""
from __future__ import annotations

import glob
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "csrc")
BUILD_DIR = os.path.join(ROOT, "hanuman_b200", "_ext_build")
EXT_NAME = "hanuman_b200_C"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr", "--expt-extended-lambda",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-DNDEBUG",
]


def sources() -> list[str]:
    srcs = sorted(glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True))
    srcs += sorted(glob.glob(os.path.join(CSRC, "**", "*.cpp"), recursive=True))
    return srcs


def so_path() -> str:
    return os.path.join(BUILD_DIR, EXT_NAME + ".so")


def build(verbose: bool = False):
    """Compile the extension (incremental) and return the loaded module."""
    import torch.utils.cpp_extension as ce

    os.makedirs(BUILD_DIR, exist_ok=True)
    # torch's arch list is bypassed: the flags above carry the only -gencode.
    os.environ["TORCH_CUDA_ARCH_LIST"] = ""
    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    mod = ce.load(
        name=EXT_NAME,
        sources=sources(),
        extra_cflags=["-O3", "-std=c++17", "-DNDEBUG"],
        extra_cuda_cflags=NVCC_FLAGS,
        extra_include_paths=[CSRC],
        extra_ldflags=["-lcuda"],
        build_directory=BUILD_DIR,
        verbose=verbose,
        with_cuda=True,
    )
    return mod


if __name__ == "__main__":
    import sys
    build(verbose="-v" in sys.argv)
    print(so_path())
