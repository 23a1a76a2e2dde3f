"""Build the sm_100a extension in place: ``python setup.py build_ext --inplace``.

The extension is compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``).
Passing ``-gencode`` in the nvcc flags makes torch skip its own arch list.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("granite_switch_b200", "csrc")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(
    glob.glob(os.path.join(CSRC, "*.cpp"))
)

nvcc_flags = [
    "-O3",
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]
if os.environ.get("GSB_PTXAS_VERBOSE") == "1":
    nvcc_flags.append("-Xptxas=-v")

setup(
    name="granite_switch_b200",
    ext_modules=[
        CUDAExtension(
            name="granite_switch_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
