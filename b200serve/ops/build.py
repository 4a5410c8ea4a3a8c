"""Build the in-tree CUDA extension for sm_100a.

The extension is compiled with ``torch.utils.cpp_extension.load`` into
``b200serve/ops/_build/`` (inside the source tree, so the built ``.so`` ships
with the repository snapshot). nvcc cross-compiles for sm_100a without a GPU.
"""

from __future__ import annotations

import glob
import os

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD_DIR = os.path.join(HERE, "_build")
EXT_NAME = "b200_ops"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xptxas", "-v",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]


def sources() -> list:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def build(verbose: bool = False):
    """Compile (incrementally, via ninja) and import the extension module."""
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load
    os.makedirs(BUILD_DIR, exist_ok=True)
    return load(
        name=EXT_NAME,
        sources=sources(),
        extra_cuda_cflags=NVCC_FLAGS,
        extra_cflags=["-O3", "-std=c++17"],
        extra_ldflags=["-lcuda"],
        build_directory=BUILD_DIR,
        verbose=verbose,
    )


def built_library_path() -> str:
    return os.path.join(BUILD_DIR, EXT_NAME + ".so")


if __name__ == "__main__":
    import sys
    build(verbose="-v" in sys.argv)
    print(built_library_path())
