"""Build the sm_100a CUDA extension of online_speculation_b200 in place.

    python setup.py build_ext --inplace

The extension is compiled for Blackwell B200 only (sm_100a); nvcc cross-compiles
it on machines without a GPU.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("online_speculation_b200", "csrc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("OSB_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-DNDEBUG",
]
CXX = ["-O3", "-std=c++17", "-DNDEBUG"]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))

setup(
    name="online_speculation_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="online_speculation_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": CXX, "nvcc": NVCC},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
