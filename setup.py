"""Builds the sm_100a extension in place: ``python setup.py build_ext --inplace``.

Every kernel is compiled for ``sm_100a`` only (``-gencode arch=compute_100a,code=sm_100a``).
torch's extension builder adds no architecture flags of its own when the nvcc flags
already name an architecture, so the flag below is the only one.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "")
ROOT = os.path.dirname(os.path.abspath(__file__))
sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + ["csrc/ext.cpp"]

nvcc_flags = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--use_fast_math",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__",
    "-Xptxas=-v" if os.environ.get("MYKB_PTXAS_VERBOSE") else "-Xptxas=-O3",
]


setup(
    name="myk_llm_b200",
    ext_modules=[
        CUDAExtension(
            name="myk_llm_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
