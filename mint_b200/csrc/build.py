"""Build the in-tree sm_100a extension ``mint_b200/_C*.so``.

    python -m mint_b200.csrc.build            # compile (ninja, parallel)
    MINT_PTXAS_VERBOSE=1 python -m mint_b200.csrc.build   # + register / spill / smem report

Every .cu file is compiled for ``-gencode arch=compute_100a,code=sm_100a`` only.
"""

from __future__ import annotations

import glob
import os
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
ROOT = CSRC.parent.parent

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--use_fast_math",
    "-DNDEBUG",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__",
    "-U__CUDA_NO_BFLOAT162_CONVERSIONS__",
]


def sources() -> list[str]:
    srcs = sorted(glob.glob(str(CSRC / "*.cu"))) + sorted(glob.glob(str(CSRC / "*.cpp")))
    return [os.path.relpath(s, ROOT) for s in srcs]


def build(verbose: bool = False) -> None:
    from setuptools import setup  # noqa: PLC0415
    from torch.utils.cpp_extension import BuildExtension, CUDAExtension  # noqa: PLC0415

    nvcc = list(NVCC_FLAGS)
    if os.environ.get("MINT_PTXAS_VERBOSE") == "1":
        nvcc.append("-Xptxas=-v")
    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    ext = CUDAExtension(
        name="mint_b200._C",
        sources=sources(),
        include_dirs=[str(CSRC)],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc},
    )
    cwd = os.getcwd()
    os.chdir(ROOT)
    try:
        setup(
            name="mint_b200_C",
            ext_modules=[ext],
            cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
            script_args=["build_ext", "--inplace", "--build-temp", str(CSRC / "_build")] + ([] if verbose else ["-q"]),
        )
    finally:
        os.chdir(cwd)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
