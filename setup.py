"""Build the kore_b200 native extension in-tree for sm_100a only.

    python setup.py build_ext --inplace
"""
import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("kore_b200", "csrc")
SM100 = ["-gencode", "arch=compute_100a,code=sm_100a"]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp")]

setup(
    name="kore_b200",
    version="0.1.0",
    packages=find_packages(include=["kore_b200*", "kore*"]),
    package_data={"kore_b200": ["data/knowledge/*.md", "eval/data/*.jsonl"]},
    ext_modules=[
        CUDAExtension(
            name="kore_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, CSRC)],
            extra_compile_args={
                "cxx": ["-O3", "-std=c++17"],
                "nvcc": SM100 + ["-O3", "-std=c++17", "-lineinfo", "--use_fast_math",
                                 "-Xptxas=-v" if os.environ.get("KORE_PTXAS_V") else "-Xptxas=-O3",
                                 "--expt-relaxed-constexpr", "-DNDEBUG"],
            },
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"console_scripts": ["kore = kore_b200.cli:main"]},
)
