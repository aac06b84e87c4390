"""Builds the sm_100a CUDA extension (`arcagi2_flashnext_dots3_b200._C`) and the host C++ extension
(`arcagi2_flashnext_dots3_b200._host`) in-tree: ``python setup.py build_ext --inplace``."""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension, CppExtension

PKG = "arcagi2_flashnext_dots3_b200"
CSRC = os.path.join(PKG, "csrc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

cuda_sources = [os.path.join(CSRC, f) for f in ("ext.cpp", "wgemm.cu")] + sorted(
    f for f in glob.glob(os.path.join(CSRC, "k_*.cu")))
cuda_sources.append(os.path.join(CSRC, "kernels.cu"))

ext = [
    CUDAExtension(
        name=f"{PKG}._C",
        sources=cuda_sources,
        include_dirs=[os.path.abspath(CSRC)],
        extra_compile_args={
            "cxx": ["-O3", "-std=c++17"],
            "nvcc": ARCH + ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
                            "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
                            "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__"],
        },
    ),
]
host_src = sorted(glob.glob(os.path.join(CSRC, "host_*.cpp")))
if host_src:
    ext.append(CppExtension(name=f"{PKG}._host", sources=host_src,
                            extra_compile_args=["-O3", "-std=c++17", "-fno-fast-math", "-ffp-contract=off"]))

setup(name=PKG, version="0.1.0", packages=[PKG], ext_modules=ext,
      cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)})
