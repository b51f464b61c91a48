"""Builds the native extension in place:  python setup.py build_ext --inplace

sm_100a only (B200): every .cu is compiled with
``-gencode arch=compute_100a,code=sm_100a``.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("build_your_own_distributed_training_b200", "csrc")
sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

setup(
    name="build_your_own_distributed_training_b200",
    ext_modules=[
        CUDAExtension(
            name="build_your_own_distributed_training_b200._C",
            sources=sources,
            extra_compile_args={
                "cxx": ["-O3", "-std=c++17"],
                "nvcc": ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
                         "-Xptxas", "-v" if os.environ.get("DTB_PTXAS_VERBOSE") else "-O3", *ARCH],
            },
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
