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


# The bounds-checked variant: every data-dependent global index (KV slots and block-table
# entries, recurrent-state slots, token and expert ids, RoPE positions) is range-checked in the
# kernel; an index out of range is recorded in a per-file error word (read with
# ``bounds_errors()``) and the access is skipped. Loaded instead of the release build when
# B200_BOUNDS_CHECK=1.
CHECKED_NAME = EXT_NAME + "_checked"
CHECKED_DIR = os.path.join(HERE, "_build_checked")
CHECK_DEFINE = "-DB200_BOUNDS_CHECK"


def _variant(checked: bool):
    return (CHECKED_NAME, CHECKED_DIR) if checked else (EXT_NAME, BUILD_DIR)


def build(verbose: bool = False, checked: bool = False):
    """Compile (incrementally, via ninja) and import the extension module."""
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load
    name, bdir = _variant(checked)
    os.makedirs(bdir, exist_ok=True)
    extra = [CHECK_DEFINE] if checked else []
    return load(
        name=name,
        sources=sources(),
        extra_cuda_cflags=NVCC_FLAGS + extra,
        extra_cflags=["-O3", "-std=c++17"] + extra,
        extra_ldflags=["-lcuda"],
        build_directory=bdir,
        verbose=verbose,
    )


def built_library_path(checked: bool = False) -> str:
    name, bdir = _variant(checked)
    return os.path.join(bdir, name + ".so")


if __name__ == "__main__":
    import sys
    chk = "--checked" in sys.argv
    build(verbose="-v" in sys.argv, checked=chk)
    print(built_library_path(chk))
