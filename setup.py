"""Build the sm_100a CUDA extension in place:  python setup.py build_ext --inplace

Every .cu file is compiled for exactly one target, sm_100a (B200), with -lineinfo; torch's own arch list is
bypassed because the -gencode flag is given explicitly.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("carbon_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr", "--expt-extended-lambda",
    "-DNDEBUG",
    "-Xptxas=-v" if os.environ.get("CARBON_PTXAS_V") else "-Xptxas=-O3",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG"]
if os.environ.get("CARBON_DEBUG_BOUNDS") == "1":       # bounds-checked debug build (see csrc/common.cuh)
    NVCC_FLAGS.append("-DCB_DEBUG_BOUNDS")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

setup(
    name="carbon_b200",
    packages=["carbon_b200"],
    ext_modules=[
        CUDAExtension(
            name="carbon_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
            libraries=["cuda"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
