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


class PinnedBuild(BuildExtension.with_options(use_ninja=True)):
    """Build, then record the digest of csrc/ the library was built from
    (b200ds/_C.srcpin, checked when the CUDA op layer is imported)."""

    def run(self):
        super().run()
        import importlib.util
        spec = importlib.util.spec_from_file_location("_srcpin", os.path.join(ROOT, "b200ds", "utils", "srcpin.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.write_pin(CSRC)


setup(
    name="b200ds",
    ext_modules=[CUDAExtension("b200ds._C", sources, include_dirs=[CSRC],
                               extra_compile_args={"cxx": CXX, "nvcc": NVCC})],
    cmdclass={"build_ext": PinnedBuild},
)
