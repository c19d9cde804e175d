"""In-tree build of the host runtime extension ``_mxrt`` (C++17, no CUDA).

It holds the checkpoint file IO (parallel pread/pwrite with CRC-32C) and the token data pipeline
(memory-mapped caches, block mixtures, packing, background prefetch). The shared object is written
to ``marin_experiments_b200/runtime/_build/`` and imported from there.
"""

from __future__ import annotations

import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD_DIR = os.path.join(HERE, "_build")
EXT_NAME = "_mxrt"


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cpp")))


def build(verbose: bool = False):
    os.makedirs(BUILD_DIR, exist_ok=True)
    from torch.utils.cpp_extension import load

    return load(name=EXT_NAME, sources=sources(), extra_cflags=["-O3", "-std=c++17", "-pthread"],
                extra_include_paths=[CSRC], extra_ldflags=["-pthread"], build_directory=BUILD_DIR,
                verbose=verbose, with_cuda=False)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print("built", os.path.join(BUILD_DIR, EXT_NAME + ".so"))
