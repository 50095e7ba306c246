"""Builds the in-tree native extension b200ds/_C (sm_100a only).

    python setup.py build_ext --inplace
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = ARCH + ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
               "-DNDEBUG", "-Xptxas=-warn-spills"]
CXX = ["-O3", "-std=c++17"]

sources = sorted(glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True))
sources += sorted(glob.glob(os.path.join(CSRC, "**", "*.cpp"), recursive=True))

setup(
    name="b200ds",
    ext_modules=[CUDAExtension("b200ds._C", sources, include_dirs=[CSRC],
                               extra_compile_args={"cxx": CXX, "nvcc": NVCC})],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
