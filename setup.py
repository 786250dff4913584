"""Builds the in-tree sm_100a CUDA extension ``verl_omni_b200._C``.

    python setup.py build_ext --inplace

Only ``-gencode arch=compute_100a,code=sm_100a`` is emitted: the kernels use tcgen05 / TMEM /
TMA instructions that exist on Blackwell (B200) only.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("verl_omni_b200", "csrc")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

nvcc_flags = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr", "--expt-extended-lambda",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
if os.environ.get("VO_PTXAS_VERBOSE"):
    nvcc_flags.append("-Xptxas=-v")
cxx_flags = ["-O3", "-std=c++17"]
if os.environ.get("VO_DEVICE_CHECKS", "0") == "1":
    # device-side bounds / range checks that record the failing line and skip the access (debug builds)
    nvcc_flags.append("-DVO_DEVICE_CHECKS")
    cxx_flags.append("-DVO_DEVICE_CHECKS")

setup(
    name="verl_omni_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="verl_omni_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, CSRC)],
            extra_compile_args={"cxx": cxx_flags, "nvcc": nvcc_flags},
            libraries=["cuda"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
