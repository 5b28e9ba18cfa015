"""Builds the native extension tempname_5090_b200._C in-tree for sm_100a.

    python setup.py build_ext --inplace

Only sm_100a (B200) code is generated; torch's own arch list is bypassed by the
explicit -gencode flag.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
SOURCES = sorted(glob.glob(os.path.join("csrc", "**", "*.cu"), recursive=True)) + sorted(
    glob.glob(os.path.join("csrc", "**", "*.cpp"), recursive=True))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
]

setup(
    name="tempname_5090_b200",
    ext_modules=[
        CUDAExtension(
            name="tempname_5090_b200._C",
            sources=SOURCES,
            include_dirs=[os.path.join(HERE, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
