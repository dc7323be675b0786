"""Build the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

All CUDA sources are compiled for Blackwell only
(``-gencode arch=compute_100a,code=sm_100a``); torch's own arch list is
bypassed because explicit ``-gencode`` flags are given.

``RO_BOUNDS_CHECK=1 python setup.py build_ext --inplace --build-temp build/checked``
builds the bounds-checked variant ``rational_optimizer_b200._C_checked``
(``-DRO_BOUNDS_CHECK``: failed index checks are recorded in a device word and
the guarded access is skipped; ``RO_CHECKED=1`` makes the package load it).
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("rational_optimizer_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17"]
CHECKED = os.environ.get("RO_BOUNDS_CHECK") == "1"
if CHECKED:
    NVCC_FLAGS.append("-DRO_BOUNDS_CHECK")
    CXX_FLAGS.append("-DRO_BOUNDS_CHECK")


def sources():
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    return [os.path.join(CSRC, "bindings.cpp")] + cu


setup(
    name="rational_optimizer_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="rational_optimizer_b200._C_checked" if CHECKED else "rational_optimizer_b200._C",
            sources=sources(),
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
