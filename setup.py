"""Build the sm_100a CUDA extension in-tree: ``python setup.py build_ext --inplace``.

Only Blackwell (sm_100a) code is generated. Passing an explicit ``-gencode`` in the
nvcc flags makes torch.utils.cpp_extension skip its own architecture list.
"""
import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17"]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(
    glob.glob(os.path.join(CSRC, "*.cpp"))
)

setup(
    name="spec_ep",
    version="0.1.0",
    packages=find_packages(include=["spec_ep", "spec_ep.*"]),
    python_requires=">=3.10",
    install_requires=["torch"],
    ext_modules=[
        CUDAExtension(
            name="spec_ep._C",
            sources=[os.path.relpath(s, ROOT) for s in sources],
            include_dirs=[CSRC],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
