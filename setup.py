"""Builds the sm_100a CUDA extension of tt_rsl_rl_b200 in-tree (``python setup.py build_ext --inplace``)."""

import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("tt_rsl_rl_b200", "ops", "csrc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# TT_RSL_RL_DEBUG_BOUNDS=1: kernels check the indices they read from memory and report bad ones in their status word
DEBUG = ["-DRL_DEBUG_BOUNDS"] if os.environ.get("TT_RSL_RL_DEBUG_BOUNDS") == "1" else []

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))

setup(
    name="tt_rsl_rl_b200",
    version="0.1.0",
    packages=find_packages(include=["tt_rsl_rl_b200", "tt_rsl_rl_b200.*"]),
    ext_modules=[
        CUDAExtension(
            name="tt_rsl_rl_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={
                "cxx": ["-O3", "-std=c++17"],
                "nvcc": ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", *ARCH, *DEBUG],
            },
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
