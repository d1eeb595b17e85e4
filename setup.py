"""Builds the sm_100a CUDA kernel library and the host-side C++ runtime in-tree.

    python setup.py build_ext --inplace

Both extensions land inside ``swarm_inference_lab_b200/`` so they travel with
the source tree; nothing is installed into site-packages.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension, CppExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
if os.environ.get("SIL_PTXAS_VERBOSE"):
    NVCC_FLAGS += ["-Xptxas", "-v"]

cuda_sources = sorted(glob.glob(os.path.join("csrc", "kernels", "*.cu"))) + [
    os.path.join("csrc", "kernels", "bindings.cpp")
]
native_sources = sorted(glob.glob(os.path.join("csrc", "native", "*.cpp")))

ext_modules = [
    CUDAExtension(
        name="swarm_inference_lab_b200._C",
        sources=cuda_sources,
        include_dirs=[os.path.join(ROOT, "csrc", "include")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        libraries=["cuda"],
    ),
]
if native_sources:
    ext_modules.append(
        CppExtension(
            name="swarm_inference_lab_b200._native",
            sources=native_sources,
            include_dirs=[os.path.join(ROOT, "csrc", "include")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"]},
            libraries=["crypto"],
        )
    )

setup(
    name="swarm_inference_lab_b200",
    version="0.1.0",
    packages=["swarm_inference_lab_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"console_scripts": ["swarm=swarm_inference_lab_b200.cli:main"]},
)
