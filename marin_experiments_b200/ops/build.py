"""In-tree build of the sm_100a CUDA extension ``_mxk``.

The extension is compiled for ``sm_100a`` only (``-gencode arch=compute_100a,code=sm_100a``)
into ``marin_experiments_b200/ops/_build/``; the loader imports the resulting ``.so`` directly
from there, so a built tree can be copied to a GPU machine and used without recompiling.
"""

from __future__ import annotations

import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD_DIR = os.path.join(HERE, "_build")
EXT_NAME = "_mxk"

CUDA_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_HALF2_OPERATORS__",
]
CXX_FLAGS = ["-O3", "-std=c++17"]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def build(verbose: bool = False):
    # torch's own arch list must not add other targets: the flags above are the only -gencode.
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.makedirs(BUILD_DIR, exist_ok=True)
    from torch.utils.cpp_extension import load

    return load(
        name=EXT_NAME,
        sources=sources(),
        extra_cuda_cflags=CUDA_FLAGS,
        extra_cflags=CXX_FLAGS,
        extra_include_paths=[CSRC],
        extra_ldflags=["-ldl"],
        build_directory=BUILD_DIR,
        verbose=verbose,
        with_cuda=True,
    )


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print("built", os.path.join(BUILD_DIR, EXT_NAME + ".so"))
