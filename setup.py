"""Build the sm_100a extension in place: ``python setup.py build_ext --inplace``.

Compiles every CUDA source for ``sm_100a`` only (tcgen05/TMA code does not
exist on other architectures) with line info for the profiler.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("dstraining_b200", "csrc")
sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

nvcc_flags = [
    "-O3",
    "-std=c++17",
    "-gencode=arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--use_fast_math",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
if os.environ.get("DST_PTXAS_VERBOSE"):
    nvcc_flags.append("-Xptxas=-v")

setup(
    name="dstraining_b200",
    ext_modules=[
        CUDAExtension(
            "dstraining_b200._C",
            sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
