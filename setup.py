"""Builds the in-tree extensions: ``nano_qwen_b200._C`` (sm_100a kernels) and
``nano_qwen_b200._runtime`` (host-side C++ runtime).

    python setup.py build_ext --inplace

Every CUDA source is compiled for ``-gencode arch=compute_100a,code=sm_100a``
only (passed in extra_cuda_cflags, which bypasses torch's own arch list).
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
SOURCES = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + [os.path.join("csrc", "bindings.cpp")]

NVCC_FLAGS = [
    "-O3",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__",
    "-U__CUDA_NO_BFLOAT162_CONVERSIONS__",
]

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 8))

setup(
    name="nano_qwen_b200",
    version="0.1.0",
    packages=["nano_qwen_b200"],
    ext_modules=[
        CUDAExtension(
            name="nano_qwen_b200._C",
            sources=SOURCES,
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        ),
        # host-side runtime (no CUDA): native data-path helpers
        CppExtension(
            name="nano_qwen_b200._runtime",
            sources=[os.path.join("csrc", "runtime", "token_reader.cpp")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"]},
        ),
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
