"""Builds the sm_100a CUDA extension in-tree: ``python setup.py build_ext --inplace``.

The extension is compiled for sm_100a only (B200).  Kernel sources are plain
CUDA; only ``bindings.cpp`` includes the torch headers.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("mini_megatron_b200", "csrc")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp"),
                                                           os.path.join(CSRC, "symm_mem.cpp")]

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_HALF2_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]

setup(
    name="mini_megatron_b200",
    ext_modules=[
        CUDAExtension(
            name="mini_megatron_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            # Link the C++ runtime that torch itself uses (the shared system
            # libstdc++).  A toolchain whose libstdc++.so link is missing would
            # otherwise fall back to libstdc++.a, and a second, static copy of
            # the C++ runtime inside the extension breaks iostream formatting
            # (every error message built by TORCH_CHECK).
            extra_link_args=["-l:libstdc++.so.6"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
