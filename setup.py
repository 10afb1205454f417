"""Build the sm_100a extension in place:  python setup.py build_ext --inplace

Produces dattri_llm_b200/_C*.so next to the Python sources, so a copy of the
tree carries its compiled kernels with it.
"""

import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]


def ext_modules():
    sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + sorted(
        glob.glob(os.path.join("csrc", "*.cpp"))
    )
    return [
        CUDAExtension(
            name="dattri_llm_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ]


setup(
    name="dattri_llm_b200",
    version="0.1.0",
    packages=find_packages(include=["dattri_llm_b200", "dattri_llm_b200.*"]),
    ext_modules=ext_modules(),
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
