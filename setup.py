"""Build the in-tree sm_100a extension: ``python setup.py build_ext --inplace``.

Every CUDA source is compiled for ``sm_100a`` only (``-gencode arch=compute_100a,code=sm_100a``),
independent of torch's own arch list.
"""
import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("llmserve_b200", "ops", "csrc")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp")]

setup(
    name="llmserve_b200",
    version="0.1.0",
    python_requires=">=3.10",
    packages=find_packages(include=["llmserve_b200", "llmserve_b200.*", "benchmarks"]),
    package_data={"benchmarks": ["suites/*.json"]},
    ext_modules=[
        CUDAExtension(
            name="llmserve_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, CSRC)],
            extra_compile_args={
                "cxx": ["-O3", "-std=c++17"],
                "nvcc": ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", *GENCODE,
                         "-Xptxas=-v" if os.environ.get("LLMSERVE_PTXAS_VERBOSE") else "-Xptxas=-O3"],
            },
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
