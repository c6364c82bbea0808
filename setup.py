"""Build the extensions in-tree:  python setup.py build_ext --inplace

`_C`: the sm_100a kernels and the domain runtime; `_host`: the CPU-side runtime library.

Only sm_100a code is generated (`-gencode arch=compute_100a,code=sm_100a`); torch's own
TORCH_CUDA_ARCH_LIST is bypassed by passing the arch flags explicitly.
"""

import os
from pathlib import Path

import pybind11
from setuptools import Extension, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = Path(__file__).resolve().parent
PKG = "hetero_cp_ringattn_b200"
CSRC = ROOT / PKG / "csrc"

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 8))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# HCP_DEBUG_BOUNDS=1: kernels also check the page ids they read from page tables (status word)
DEBUG = ["-DHCP_DEBUG_BOUNDS=1"] if os.environ.get("HCP_DEBUG_BOUNDS") == "1" else []
NVCC_FLAGS = ARCH + DEBUG + ["-O3", "-std=c++17", "-lineinfo", "--use_fast_math", "-Xptxas=-v",
                     "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
                     "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT162_OPERATORS__",
                     "--expt-relaxed-constexpr"]
SOURCES = [
    "bindings.cpp",
    "core/runtime.cu",
    "kernels/gemm_sm100.cu",
    "kernels/attn_fwd_sm100.cu",
    "kernels/elementwise.cu",
    "kernels/decode.cu",
]

# host runtime library (no CUDA, no libtorch): layouts, capacity, schedule, pages, scheduler
HOST_SOURCES = ["layout.cpp", "capacity.cpp", "schedule.cpp", "pages.cpp", "scheduler.cpp",
                "protocol.cpp", "ref_attention.cpp", "host_bindings.cpp"]

setup(
    name=PKG,
    version="0.1.0",
    packages=[PKG],
    ext_modules=[
        CUDAExtension(
            name=f"{PKG}._C",
            sources=[str(CSRC / s) for s in SOURCES],
            include_dirs=[str(CSRC / "include"), str(CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        ),
        Extension(
            name=f"{PKG}._host",
            sources=[str(CSRC / "host" / s) for s in HOST_SOURCES],
            include_dirs=[str(CSRC / "host"), pybind11.get_include()],
            extra_compile_args=["-O3", "-std=c++17", "-fvisibility=hidden", "-Wall"],
            language="c++",
        ),
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
