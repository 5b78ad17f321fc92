"""Build the vlmrl sm_100a CUDA extension in-tree: ``python setup.py build_ext --inplace``."""

import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
SOURCES = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + sorted(glob.glob(os.path.join("csrc", "*.cpp")))

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-Xptxas=-warn-spills",
]

setup(
    name="vlmrl",
    version="0.1.0",
    packages=find_packages(include=["vlmrl", "vlmrl.*"]),
    package_data={"vlmrl.assets": ["imgs/*.png"]},
    ext_modules=[
        CUDAExtension(
            name="vlmrl._C",
            sources=SOURCES,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
